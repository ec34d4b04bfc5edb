// comm.cc -- row-shard planning and the multi-process sharded linear
// (include/hexir_b200/comm.h).

#include <algorithm>
#include <cstring>
#include <new>
#include <string>

#include "cuda_driver.h"
#include "hexir_b200/comm.h"
#include "hexir_b200/kernels.h"
#include "kernel_lib.h"
#include "nccl_shim.h"

using namespace hexir;

namespace {
// A rank's output rows leave for the root in up to kGatherChunks pieces of
// geometrically shrinking size (1/2, 1/4, 1/8, 1/16, 1/16 of its rows), so
// every transfer but the last hides behind the GEMM of the next piece and the
// exposed last one is small.  Pieces keep >= kMinChunkRows rows.
constexpr uint32_t kGatherChunks = 5;
constexpr uint64_t kMinChunkRows = 256;

// Piece `i` of `rows` rows: [*begin, *begin + *count).  Returns the number of
// pieces.  Deterministic, so the root computes every peer's pieces.
uint32_t gather_piece(uint64_t rows, uint32_t i, uint64_t *begin,
                      uint64_t *count) {
  uint32_t pieces = 1;
  uint64_t bounds[kGatherChunks + 1] = {0};
  uint64_t done = 0;
  for (uint32_t p = 0; p < kGatherChunks; ++p) {
    const uint64_t left = rows - done;
    uint64_t take = p + 1 == kGatherChunks ? left : left / 2;
    // Round to 128-row tiles; the remainder must stay a worthwhile piece.
    take = (take / 128) * 128;
    if (take < kMinChunkRows || left - take < kMinChunkRows)
      take = left;
    done += take;
    bounds[p + 1] = done;
    pieces = p + 1;
    if (done == rows)
      break;
  }
  if (i >= pieces) {
    *begin = rows;
    *count = 0;
  } else {
    *begin = bounds[i];
    *count = bounds[i + 1] - bounds[i];
  }
  return pieces;
}
}  // namespace

struct hexir_comm_t {
  ncclComm_t comm = nullptr;
  int nranks = 0;
  int rank = 0;
  int ordinal = 0;
  CUstream gather_stream = nullptr;  // row sends / receives
  CUevent chunk_done[kGatherChunks] = {};
  CUevent gather_done = nullptr;
};

extern "C" {

hexir_status_t hexir_shard_rows(uint64_t rows, uint32_t shards, uint32_t index,
                                uint64_t *begin, uint64_t *count) {
  if (!begin || !count || shards == 0 || index >= shards)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  const uint64_t base = rows / shards, extra = rows % shards;
  *begin = index * base + (index < extra ? index : extra);
  *count = base + (index < extra ? 1 : 0);
  return HEXIR_OK;
}

hexir_status_t hexir_comm_unique_id(void *id, size_t size) {
  if (!id || size < sizeof(ncclUniqueId))
    return HEXIR_ERROR_INVALID_ARGUMENT;
  const Nccl &n = nccl();
  if (!n.ok) {
    set_last_error(n.error);
    return HEXIR_ERROR_DEVICE;
  }
  ncclUniqueId uid;
  ncclResult_t r = n.GetUniqueId(&uid);
  if (r != ncclSuccess) {
    set_last_error(nccl_message("ncclGetUniqueId", r));
    return HEXIR_ERROR_DEVICE;
  }
  std::memcpy(id, &uid, sizeof(uid));
  return HEXIR_OK;
}

hexir_status_t hexir_comm_init_rank(const void *id, size_t size, int nranks,
                                    int rank, int ordinal, hexir_comm_t **out) {
  if (!id || !out || size < sizeof(ncclUniqueId) || nranks < 1 || rank < 0 ||
      rank >= nranks)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  *out = nullptr;
  const Nccl &n = nccl();
  if (!n.ok) {
    set_last_error(n.error);
    return HEXIR_ERROR_DEVICE;
  }
  std::string error;
  DeviceState *dev = device_state(ordinal, &error);
  if (!dev) {
    set_last_error(error);
    return HEXIR_ERROR_DEVICE;
  }
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  auto *comm = new (std::nothrow) hexir_comm_t;
  if (!comm)
    return HEXIR_ERROR_OUT_OF_MEMORY;
  ContextGuard guard(dev->context);
  ncclResult_t r = n.CommInitRank(&comm->comm, nranks, uid, rank);
  if (r != ncclSuccess) {
    set_last_error(nccl_message("ncclCommInitRank", r));
    delete comm;
    return HEXIR_ERROR_DEVICE;
  }
  comm->nranks = nranks;
  comm->rank = rank;
  comm->ordinal = ordinal;
  const Driver &d = driver();
  CUresult cr = d.StreamCreate(&comm->gather_stream, CU_STREAM_NON_BLOCKING);
  for (uint32_t i = 0; cr == CUDA_SUCCESS && i < kGatherChunks; ++i)
    cr = d.EventCreate(&comm->chunk_done[i], CU_EVENT_DISABLE_TIMING);
  if (cr == CUDA_SUCCESS)
    cr = d.EventCreate(&comm->gather_done, CU_EVENT_DISABLE_TIMING);
  if (cr != CUDA_SUCCESS) {
    set_last_error(cuda_message("gather stream set-up", cr));
    hexir_comm_release(comm);
    return HEXIR_ERROR_DEVICE;
  }
  *out = comm;
  return HEXIR_OK;
}

void hexir_comm_release(hexir_comm_t *comm) {
  if (!comm)
    return;
  std::string error;
  DeviceState *dev = device_state(comm->ordinal, &error);
  if (dev) {
    ContextGuard guard(dev->context);
    const Driver &d = driver();
    if (comm->gather_stream) {
      d.StreamSynchronize(comm->gather_stream);
      d.StreamDestroy(comm->gather_stream);
    }
    for (CUevent ev : comm->chunk_done)
      if (ev)
        d.EventDestroy(ev);
    if (comm->gather_done)
      d.EventDestroy(comm->gather_done);
  }
  if (comm->comm && nccl().ok)
    nccl().CommDestroy(comm->comm);
  delete comm;
}

int hexir_comm_rank(const hexir_comm_t *comm) { return comm ? comm->rank : -1; }
int hexir_comm_size(const hexir_comm_t *comm) {
  return comm ? comm->nranks : 0;
}

hexir_status_t hexir_sharded_linear_f64(hexir_comm_t *comm, const double *a_rows,
                                        double *w, double *c, uint32_t m,
                                        uint32_t n, uint32_t k, uint32_t flags,
                                        void *stream) {
  if (!comm || !w || !c)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  const Nccl &nc = nccl();
  std::string error;
  DeviceState *dev = device_state(comm->ordinal, &error);
  if (!dev) {
    set_last_error(error);
    return HEXIR_ERROR_DEVICE;
  }
  KernelLib *lib = embedded_library(dev, &error);
  if (!lib) {
    set_last_error(error);
    return HEXIR_ERROR_DEVICE;
  }
  ContextGuard guard(dev->context);
  CUstream s = static_cast<CUstream>(stream);
  const uint32_t ranks = static_cast<uint32_t>(comm->nranks);
  uint64_t begin = 0, rows = 0;
  hexir_shard_rows(m, ranks, static_cast<uint32_t>(comm->rank), &begin, &rows);

  // 1. Weight from the root to everyone, over NVLink.
  ncclResult_t r = nc.Broadcast(w, w, static_cast<size_t>(k) * n, ncclDouble, 0,
                                comm->comm, reinterpret_cast<cudaStream_t>(s));
  if (r != ncclSuccess) {
    set_last_error(nccl_message("ncclBroadcast", r));
    return HEXIR_ERROR_DEVICE;
  }
  // 2. This rank's rows in up to kGatherChunks pieces; the root writes
  //    straight into its part of c.  3. Each finished piece goes to the root
  //    on the gather stream while the next piece computes.  Every rank splits
  //    its rows by the same rule, so the root knows each peer's pieces.
  const Driver &d = driver();
  uint64_t ignore_b = 0, ignore_c = 0;
  const uint32_t my_chunks = rows ? gather_piece(rows, 0, &ignore_b, &ignore_c) : 0;
  uint32_t max_chunks = 0;
  for (uint32_t peer = 0; peer < ranks; ++peer) {
    uint64_t pb = 0, pr = 0;
    hexir_shard_rows(m, ranks, peer, &pb, &pr);
    if (pr)
      max_chunks = std::max(max_chunks, gather_piece(pr, 0, &ignore_b, &ignore_c));
  }
  cudaStream_t gs = reinterpret_cast<cudaStream_t>(comm->gather_stream);
  for (uint32_t i = 0; i < max_chunks; ++i) {
    if (i < my_chunks) {
      uint64_t cb = 0, cr = 0;
      gather_piece(rows, i, &cb, &cr);
      if (cr) {
        hexir_status_t st = launch_matmul(
            dev, lib, a_rows + cb * k, w, c + cb * n, static_cast<uint32_t>(cr),
            n, k, flags & HEXIR_MATMUL_RELU, s, &error);
        if (st != HEXIR_OK) {
          set_last_error(error);
          return st;
        }
      }
    }
    if (ranks == 1)
      continue;
    d.EventRecord(comm->chunk_done[i], s);
    d.StreamWaitEvent(comm->gather_stream, comm->chunk_done[i], 0);
    nc.GroupStart();
    if (comm->rank == 0) {
      for (uint32_t peer = 1; peer < ranks; ++peer) {
        uint64_t pb = 0, pr = 0;
        hexir_shard_rows(m, ranks, peer, &pb, &pr);
        uint64_t cb = 0, cr = 0;
        if (!pr)
          continue;
        gather_piece(pr, i, &cb, &cr);
        if (cr)
          nc.Recv(c + (pb + cb) * n, cr * n, ncclDouble, static_cast<int>(peer),
                  comm->comm, gs);
      }
    } else if (i < my_chunks) {
      uint64_t cb = 0, cr = 0;
      gather_piece(rows, i, &cb, &cr);
      if (cr)
        nc.Send(c + cb * n, cr * n, ncclDouble, 0, comm->comm, gs);
    }
    r = nc.GroupEnd();
    if (r != ncclSuccess) {
      set_last_error(nccl_message("ncclGroupEnd (row gather)", r));
      return HEXIR_ERROR_DEVICE;
    }
  }
  if (ranks > 1) {
    // The caller's stream completes only after the gather.
    d.EventRecord(comm->gather_done, comm->gather_stream);
    d.StreamWaitEvent(s, comm->gather_done, 0);
  }
  return HEXIR_OK;
}

}  // extern "C"
