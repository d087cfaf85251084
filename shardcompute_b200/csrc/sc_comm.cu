// NCCL over NVLink / NVSwitch in place of the reference's asyncio-TCP ring
// collectives (collectives/all_reduce.py:58-193, all_gather.py:54-162).
// One communicator per process (one process per GPU); the 128-byte unique id
// travels over the host store chosen by the Python layer.
//
// Failure handling: collectives are enqueued on the caller's stream; a host
// watchdog calls sc_comm_poll (ncclCommGetAsyncError) and, past its deadline,
// sc_comm_abort, which unblocks ranks stuck waiting for a dead peer.
#include <nccl.h>
#include <string.h>

#include "sc_common.cuh"

namespace sc {

struct Comm {
  ncclComm_t nccl;
  int world;
  int rank;
};

static ncclDataType_t nccl_type(int dt, bool* ok) {
  *ok = true;
  switch (dt) {
    case SC_F16: return ncclFloat16;
    case SC_F32: return ncclFloat32;
    case SC_I32: return ncclInt32;
    case SC_U8: return ncclUint8;
  }
  *ok = false;
  return ncclFloat32;
}

static ncclRedOp_t nccl_op(int op, bool* ok) {
  *ok = true;
  switch (op) {
    case SC_OP_SUM: return ncclSum;
    case SC_OP_MAX: return ncclMax;
    case SC_OP_MIN: return ncclMin;
    case SC_OP_AVG: return ncclAvg;
  }
  *ok = false;
  return ncclSum;
}

static int nccl_status(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return SC_OK;
  set_error("%s: NCCL error %d (%s)", what, (int)r, ncclGetErrorString(r));
  return SC_ERR_NCCL;
}

}  // namespace sc

extern "C" {

int sc_comm_unique_id(void* uid_out, size_t uid_bytes) {
  SC_REQUIRE(uid_out && uid_bytes >= sizeof(ncclUniqueId), SC_ERR_ARG, "comm_unique_id: need %zu bytes",
             sizeof(ncclUniqueId));
  ncclUniqueId id;
  int st = sc::nccl_status(ncclGetUniqueId(&id), "ncclGetUniqueId");
  if (st != SC_OK) return st;
  memcpy(uid_out, &id, sizeof(id));
  return SC_OK;
}

int sc_comm_init(const void* uid, size_t uid_bytes, int world, int rank, void** comm_out) {
  SC_REQUIRE(uid && comm_out && uid_bytes >= sizeof(ncclUniqueId), SC_ERR_ARG, "comm_init: bad arguments");
  SC_REQUIRE(world >= 1 && rank >= 0 && rank < world, SC_ERR_SHAPE, "comm_init: rank %d of %d", rank, world);
  ncclUniqueId id;
  memcpy(&id, uid, sizeof(id));
  ncclComm_t c;
  int st = sc::nccl_status(ncclCommInitRank(&c, world, id, rank), "ncclCommInitRank");
  if (st != SC_OK) return st;
  sc::Comm* h = new sc::Comm{c, world, rank};
  *comm_out = h;
  return SC_OK;
}

int sc_comm_destroy(void* comm) {
  if (!comm) return SC_OK;
  sc::Comm* h = static_cast<sc::Comm*>(comm);
  int st = sc::nccl_status(ncclCommDestroy(h->nccl), "ncclCommDestroy");
  delete h;
  return st;
}

int sc_comm_abort(void* comm) {
  if (!comm) return SC_OK;
  sc::Comm* h = static_cast<sc::Comm*>(comm);
  int st = sc::nccl_status(ncclCommAbort(h->nccl), "ncclCommAbort");
  delete h;
  return st;
}

int sc_comm_poll(void* comm, int* async_error) {
  SC_REQUIRE(comm && async_error, SC_ERR_ARG, "comm_poll: null pointer");
  ncclResult_t r = ncclSuccess;
  int st = sc::nccl_status(ncclCommGetAsyncError(static_cast<sc::Comm*>(comm)->nccl, &r), "ncclCommGetAsyncError");
  *async_error = (int)r;
  return st;
}

int sc_allreduce(const void* send, void* recv, size_t count, int dtype, int op, void* comm, cudaStream_t stream) {
  SC_REQUIRE(comm && send && recv, SC_ERR_ARG, "allreduce: null pointer");
  bool ok1, ok2;
  const ncclDataType_t t = sc::nccl_type(dtype, &ok1);
  const ncclRedOp_t o = sc::nccl_op(op, &ok2);
  SC_REQUIRE(ok1 && ok2, SC_ERR_ARG, "allreduce: dtype %d / op %d", dtype, op);
  if (count == 0) return SC_OK;
  return sc::nccl_status(ncclAllReduce(send, recv, count, t, o, static_cast<sc::Comm*>(comm)->nccl, stream),
                         "ncclAllReduce");
}

int sc_allgather(const void* send, void* recv, size_t count_per_rank, int dtype, void* comm, cudaStream_t stream) {
  SC_REQUIRE(comm && send && recv, SC_ERR_ARG, "allgather: null pointer");
  bool ok;
  const ncclDataType_t t = sc::nccl_type(dtype, &ok);
  SC_REQUIRE(ok, SC_ERR_ARG, "allgather: dtype %d", dtype);
  if (count_per_rank == 0) return SC_OK;
  return sc::nccl_status(ncclAllGather(send, recv, count_per_rank, t, static_cast<sc::Comm*>(comm)->nccl, stream),
                         "ncclAllGather");
}

int sc_broadcast(const void* send, void* recv, size_t count, int dtype, int root, void* comm, cudaStream_t stream) {
  SC_REQUIRE(comm && recv, SC_ERR_ARG, "broadcast: null pointer");
  bool ok;
  const ncclDataType_t t = sc::nccl_type(dtype, &ok);
  SC_REQUIRE(ok, SC_ERR_ARG, "broadcast: dtype %d", dtype);
  if (count == 0) return SC_OK;
  return sc::nccl_status(ncclBroadcast(send, recv, count, t, root, static_cast<sc::Comm*>(comm)->nccl, stream),
                         "ncclBroadcast");
}

// Point-to-point: one rank's send matches the peer's recv of the same count
// and dtype (Communicator.send / recv, collectives/communicator.py:520-561;
// the pipeline stage transfers of worker/executor.py:376-479).
int sc_send(const void* buf, size_t count, int dtype, int peer, void* comm, cudaStream_t stream) {
  SC_REQUIRE(comm && buf, SC_ERR_ARG, "send: null pointer");
  bool ok;
  const ncclDataType_t t = sc::nccl_type(dtype, &ok);
  SC_REQUIRE(ok, SC_ERR_ARG, "send: dtype %d", dtype);
  if (count == 0) return SC_OK;
  return sc::nccl_status(ncclSend(buf, count, t, peer, static_cast<sc::Comm*>(comm)->nccl, stream), "ncclSend");
}

int sc_recv(void* buf, size_t count, int dtype, int peer, void* comm, cudaStream_t stream) {
  SC_REQUIRE(comm && buf, SC_ERR_ARG, "recv: null pointer");
  bool ok;
  const ncclDataType_t t = sc::nccl_type(dtype, &ok);
  SC_REQUIRE(ok, SC_ERR_ARG, "recv: dtype %d", dtype);
  if (count == 0) return SC_OK;
  return sc::nccl_status(ncclRecv(buf, count, t, peer, static_cast<sc::Comm*>(comm)->nccl, stream), "ncclRecv");
}

}  // extern "C"
