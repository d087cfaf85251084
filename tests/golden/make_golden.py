"""Generate the golden fixtures in this directory (run from the repo root:
``python tests/golden/make_golden.py``).

``affine_kat.npz`` -- known answers written from the format definition, not
from the oracle: hand-built words holding every 4-bit code at every nibble
position and every 8-bit code at every byte position, with the codes they
must unpack to, and dequantized values for scales/biases whose products are
exact in fp16 (including a negative scale, zero scale, and the fp16 extremes
of the code range).

``oracle_small.npz`` -- seeded cases computed by the CPU oracle (pack layout,
quantize, dequantize, quantized_matmul, vocab-split embedding, a 2-layer
quantized Llama forward at TP 1 and TP 2, and greedy tokens).  They freeze the
oracle's outputs so both the oracle and the CUDA path are checked against the
same committed numbers.

The reference (MLX) cannot run in this environment, so no fixture comes from
the reference itself; parity of the quantized arithmetic with MLX is unpinned.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)


def kat():
    out = {}
    # 4-bit: word k (0..15) holds code (k + j) % 16 at nibble j -> every code at every position
    codes4 = np.array([[(k + j) % 16 for j in range(8)] for k in range(16)], dtype=np.uint8)
    words4 = np.array([sum(int(c) << (4 * j) for j, c in enumerate(row)) for row in codes4], dtype=np.uint32)
    out["w4_words"], out["w4_codes"] = words4.reshape(2, 8), codes4.reshape(2, 64)
    # 8-bit: 64 words x 4 bytes cover all 256 codes at each byte position
    base = np.array([[(4 * k + 64 * j) % 256 for j in range(4)] for k in range(64)], dtype=np.int64)
    codes8 = np.concatenate([(base + d) % 256 for d in range(4)]).astype(np.uint8)
    words8 = np.array([sum(int(c) << (8 * j) for j, c in enumerate(row)) for row in codes8], dtype=np.uint32)
    out["w8_words"], out["w8_codes"] = words8.reshape(4, 64), codes8.reshape(4, 256)
    # dequant with exact fp16 products: (scale, bias) per group of 32 along the 64 codes of each 4-bit row
    sc = np.array([[0.5, -0.25], [0.0, 2.0]], dtype=np.float16)
    bi = np.array([[-1.0, 3.0], [7.5, -16.0]], dtype=np.float16)
    q = codes4.reshape(2, 64).astype(np.float64)
    out["w4_scales_g32"], out["w4_biases_g32"] = sc, bi
    out["w4_dequant_g32"] = (np.repeat(sc.astype(np.float64), 32, 1) * q + np.repeat(bi.astype(np.float64), 32, 1)
                             ).astype(np.float16)
    return out


def oracle_cases():
    from oracle import mlx_affine as qa
    from oracle import sharder as osh
    from oracle import synth, tp

    rng = np.random.Generator(np.random.PCG64(2024))
    out = {}
    for bits in (4, 8):
        for g in (32, 64, 128):
            w = (rng.standard_normal((48, 256)) * 0.02).astype(np.float16)
            w[3, :g] = np.float16(0.0125)  # constant group: scale 0, q 0
            wq, s, b = qa.quantize(w, g, bits)
            x = rng.standard_normal((3, 256)).astype(np.float16)
            key = f"b{bits}_g{g}"
            out[f"{key}_w"], out[f"{key}_wq"], out[f"{key}_s"], out[f"{key}_b"] = w, wq, s, b
            out[f"{key}_deq"] = qa.dequantize(wq, s, b, g, bits)
            out[f"{key}_x"] = x
            out[f"{key}_y"] = qa.quantized_matmul(x, wq, s, b, g, bits)
    # vocab-split quantized embedding, world 4
    cfg = tp.LlamaShape(vocab_size=256, hidden_size=128, num_layers=1, num_heads=2, num_kv_heads=2,
                        intermediate_size=256)
    tab = (rng.standard_normal((256, 128)) * 0.02).astype(np.float16)
    ewq, es, eb = qa.quantize(tab, 64, 4)
    ids = rng.integers(0, 256, size=(2, 7))
    out["emb_wq"], out["emb_s"], out["emb_b"], out["emb_ids"] = ewq, es, eb, ids
    for world in (1, 4):
        for r in range(world):
            sh = dict(zip(("model.embed_tokens.weight", "model.embed_tokens.scales", "model.embed_tokens.biases"),
                          osh.shard_quantized("model.embed_tokens.weight", ewq, es, eb, world, r)))
            out[f"emb_w{world}_r{r}"] = tp.embed_rank(ids, sh, cfg, world, r)
    # a 2-layer quantized Llama at TP 1 and TP 2
    shape = synth.tiny_shape(vocab_size=512, hidden_size=256, num_layers=2, num_heads=4, num_kv_heads=2,
                             intermediate_size=512)
    full = synth.checkpoint(shape, seed=17)
    prompt = rng.integers(0, shape.vocab_size, size=(1, 6))
    out["llama_prompt"] = prompt
    for world in (1, 2):
        shards = [osh.shard_weights(full, world, r) for r in range(world)]
        m = tp.TPModel(shards, shape, max_len=64)
        logits, hidden = m.forward(prompt, return_hidden=True)
        out[f"llama_tp{world}_logits"] = logits.astype(np.float32)
        out[f"llama_tp{world}_hidden"] = np.stack(hidden).astype(np.float32)
        out[f"llama_tp{world}_greedy"] = m.generate(prompt, 6)
    return out


def main():
    np.savez_compressed(os.path.join(HERE, "affine_kat.npz"), **kat())
    np.savez_compressed(os.path.join(HERE, "oracle_small.npz"), **oracle_cases())
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
