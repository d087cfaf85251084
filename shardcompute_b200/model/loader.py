"""Direct safetensors -> device loading of a rank's shard.

Replaces the reference's per-tensor load path (``model/loader.py:106-423``:
``safetensors`` -> numpy -> ``mx.array`` one tensor at a time).  Here the
file's header is parsed once, the tensor bytes stream from disk through two
pinned host buffers (a chunk is read while the previous one is copied) into
ONE device allocation, each tensor at a 256-byte aligned offset (the tensor
maps and bulk copies of the kernels want 16-byte aligned bases), and every
tensor is returned as a view of that allocation with its own dtype and shape.
Packed ``U32`` words come back as ``int32`` (the same bytes; the kernels read
them as 32-bit words).

The safetensors format: an 8-byte little-endian header length, a JSON header
``{name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__": {...}}``
and the tensors' bytes, offsets relative to the end of the header.
"""

from __future__ import annotations

import json
import os
import struct
from typing import Dict, Iterable, List, Optional, Tuple

import torch

_DTYPES = {
    "F16": torch.float16, "BF16": torch.bfloat16, "F32": torch.float32, "F64": torch.float64,
    "U32": torch.int32, "I32": torch.int32, "I64": torch.int64, "I16": torch.int16, "U8": torch.uint8,
    "I8": torch.int8, "BOOL": torch.bool,
}
_ALIGN = 256


def read_header(path: str) -> Tuple[Dict[str, dict], int]:
    """(tensor entries by name, byte offset of the data region)."""
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"{path}: not a safetensors file (short header length)")
        n = struct.unpack("<Q", raw)[0]
        head = f.read(n)
        if len(head) != n:
            raise ValueError(f"{path}: truncated header")
    entries = json.loads(head.decode("utf-8"))
    entries.pop("__metadata__", None)
    for name, e in entries.items():
        if e["dtype"] not in _DTYPES:
            raise ValueError(f"{path}: tensor {name} has unsupported dtype {e['dtype']}")
        b, end = e["data_offsets"]
        esz = torch.empty((), dtype=_DTYPES[e["dtype"]]).element_size()
        count = 1
        for d in e["shape"]:
            count *= d
        if end - b != count * esz:
            raise ValueError(f"{path}: tensor {name} spans {end - b} bytes, shape needs {count * esz}")
    return entries, 8 + n


def load_safetensors(path: str, device, names: Optional[Iterable[str]] = None,
                     chunk_bytes: int = 256 << 20) -> Dict[str, torch.Tensor]:
    """Every tensor of ``path`` (or those in ``names``) on ``device``, as views
    of one allocation.  ``chunk_bytes``: size of each pinned staging buffer."""
    device = torch.device(device)
    entries, data0 = read_header(path)
    want = list(entries) if names is None else list(names)
    missing = [n for n in want if n not in entries]
    if missing:
        raise KeyError(f"{path}: missing tensors {missing[:4]}")
    # file order, so the reads are sequential
    order = sorted(want, key=lambda n: entries[n]["data_offsets"][0])
    dst: Dict[str, int] = {}
    total = 0
    for n in order:
        dst[n] = total
        b, e = entries[n]["data_offsets"]
        total += (e - b + _ALIGN - 1) // _ALIGN * _ALIGN
    buf = torch.empty(max(total, 1), dtype=torch.uint8, device=device)
    cuda = device.type == "cuda"
    chunk_bytes = max(1 << 16, int(chunk_bytes))
    stage = [torch.empty(chunk_bytes, dtype=torch.uint8, pin_memory=cuda) for _ in range(2 if cuda else 1)]
    done: List[Optional[torch.cuda.Event]] = [None] * len(stage)
    # pieces: (file offset, bytes, device offset), in file order, cut at chunk_bytes
    pieces = []
    for n in order:
        b, e = entries[n]["data_offsets"]
        off = 0
        while off < e - b:
            m = min(chunk_bytes, e - b - off)
            pieces.append((data0 + b + off, m, dst[n] + off))
            off += m
    stream = torch.cuda.Stream(device=device) if cuda else None
    with open(path, "rb", buffering=0) as f:
        i, k = 0, 0
        while i < len(pieces):
            # one chunk: consecutive pieces that fit the staging buffer
            j, used = i, 0
            while j < len(pieces) and used + pieces[j][1] <= chunk_bytes:
                used += pieces[j][1]
                j += 1
            sb = stage[k % len(stage)]
            if done[k % len(stage)] is not None:
                done[k % len(stage)].synchronize()  # its previous copies have left the buffer
            pos = 0
            for (fo, m, _) in pieces[i:j]:
                f.seek(fo)
                view = memoryview(sb.numpy()).cast("B")[pos:pos + m]
                got = f.readinto(view)
                if got != m:
                    raise IOError(f"{path}: short read at offset {fo}")
                pos += m
            if cuda:
                with torch.cuda.stream(stream):
                    pos = 0
                    for (_, m, do) in pieces[i:j]:
                        buf[do:do + m].copy_(sb[pos:pos + m], non_blocking=True)
                        pos += m
                    ev = torch.cuda.Event()
                    ev.record(stream)
                    done[k % len(stage)] = ev
            else:
                pos = 0
                for (_, m, do) in pieces[i:j]:
                    buf[do:do + m].copy_(sb[pos:pos + m])
                    pos += m
            i, k = j, k + 1
    if cuda:
        stream.synchronize()
    out = {}
    for n in want:
        e = entries[n]
        b, end = e["data_offsets"]
        t = buf[dst[n]:dst[n] + (end - b)].view(_DTYPES[e["dtype"]])
        out[n] = t.view(e["shape"]) if e["shape"] else t.view(())
    return out


def load_rank_shard(shard_dir: str, rank: int, device) -> Dict[str, torch.Tensor]:
    """``shard_dir/rank_{rank}/model.safetensors`` (the layout ``WeightSharder``
    and the reference's ``model/sharder.py:318-364`` write) on ``device``."""
    path = os.path.join(shard_dir, f"rank_{rank}", "model.safetensors")
    if not os.path.exists(path):
        raise FileNotFoundError(path)
    return load_safetensors(path, device)
