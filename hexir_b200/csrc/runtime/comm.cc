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
constexpr uint32_t kGatherChunks = HEXIR_SHARD_MAX_GATHER_PIECES;
// hexir_sharded_linear_host_f64 moves a rank's rows through its host link
// in kHostChunks row chunks: 1/8, 1/4, 1/4, 1/4, 1/8 of the rows (whole
// 128-row tiles), so the first upload that compute waits for and the last
// download left after it are each an eighth.
constexpr uint32_t kHostChunks = 5;
void host_chunk(uint64_t rows, uint32_t i, uint64_t *begin, uint64_t *count) {
  static const uint32_t eighths[kHostChunks + 1] = {0, 1, 3, 5, 7, 8};
  auto bound = [&](uint32_t j) {
    return j == kHostChunks ? rows : (rows * eighths[j] / 8) / 128 * 128;
  };
  *begin = bound(i);
  *count = bound(i + 1) - *begin;
}
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

// Where the root's output lives, as the peers need it to store their rows
// there directly: a CUDA IPC handle of the allocation holding c and c's
// offset in it.  Broadcast from the root every call (its c may change).
struct RootOutput {
  uint32_t magic;
  uint32_t valid;  // 0: this call gathers with NCCL
  uint64_t offset;
  CUipcMemHandle handle;
};
constexpr uint32_t kRootOutputMagic = 0x4f525848u;  // "HXRO"
constexpr size_t kDescBytes = 128;
static_assert(sizeof(RootOutput) <= kDescBytes, "descriptor too large");
// Pinned descriptor slots, reused round robin once their copy has finished.
constexpr uint32_t kDescSlots = 8;
// Root allocations a peer keeps mapped.
constexpr size_t kMaxMapped = 4;

struct MappedOutput {
  CUipcMemHandle handle;
  CUdeviceptr base;
  uint64_t last_use;
};
}  // namespace

struct hexir_comm_t {
  ncclComm_t comm = nullptr;
  int nranks = 0;
  int rank = 0;
  int ordinal = 0;
  CUstream gather_stream = nullptr;  // weight pieces, row sends / receives
  CUevent chunk_done[kGatherChunks] = {};
  CUevent gather_done = nullptr;
  // The weight broadcast on the side stream: its start (after the caller's
  // queued work), each piece landing, the whole weight landed.
  CUevent w_start = nullptr, w_piece[2] = {}, w_done = nullptr;
  // Direct row stores into the root's c (all ranks on one host, IPC works).
  bool direct = false;
  // Device scratch: the root's output descriptor [kDescBytes], then the
  // failure word -- nonzero once any rank's part of a sharded call failed
  // since the last hexir_comm_synchronize (every call max-reduces it).
  CUdeviceptr scratch = 0;
  RootOutput *desc_host = nullptr;  // pinned [kDescSlots]
  CUevent desc_done[kDescSlots] = {};
  uint32_t desc_next = 0;
  MappedOutput mapped[kMaxMapped] = {};
  size_t mapped_count = 0;
  uint64_t calls = 0;
  // hexir_sharded_linear_host_f64: streams for this GPU's host link (one
  // each way), its events, and device workspace kept between calls.
  CUstream up_stream = nullptr, down_stream = nullptr;
  CUstream side_stream = nullptr;  // odd row chunks (their tails overlap)
  CUevent down_done = nullptr;
  CUdeviceptr a_dev = 0, w_dev = 0, c_dev = 0;
  size_t a_bytes = 0, w_bytes = 0, c_bytes = 0;
};

namespace {

hexir_status_t comm_fail(const std::string &message) {
  set_last_error(message);
  return HEXIR_ERROR_DEVICE;
}

// The pinned descriptor slot for this call, once its previous copy is done.
RootOutput *next_desc(hexir_comm_t *comm, CUevent *done) {
  const uint32_t i = comm->desc_next++ % kDescSlots;
  driver().EventSynchronize(comm->desc_done[i]);
  *done = comm->desc_done[i];
  return &comm->desc_host[i];
}

// The root's allocation `handle` mapped into this peer, opened on first use.
// At most kMaxMapped stay open; the least recently used one is closed after
// the context has finished every kernel that could store through it.
hexir_status_t map_root_output(hexir_comm_t *comm, const CUipcMemHandle &handle,
                               CUdeviceptr *base) {
  const Driver &d = driver();
  ++comm->calls;
  for (size_t i = 0; i < comm->mapped_count; ++i)
    if (std::memcmp(&comm->mapped[i].handle, &handle, sizeof(handle)) == 0) {
      comm->mapped[i].last_use = comm->calls;
      *base = comm->mapped[i].base;
      return HEXIR_OK;
    }
  size_t slot = comm->mapped_count;
  if (slot == kMaxMapped) {
    slot = 0;
    for (size_t i = 1; i < kMaxMapped; ++i)
      if (comm->mapped[i].last_use < comm->mapped[slot].last_use)
        slot = i;
    CUresult r = d.CtxSynchronize();
    if (r == CUDA_SUCCESS)
      r = d.IpcCloseMemHandle(comm->mapped[slot].base);
    if (r != CUDA_SUCCESS)
      return comm_fail(cuda_message("closing a mapping of the root's output", r));
    --comm->mapped_count;
    comm->mapped[slot] = comm->mapped[comm->mapped_count];
    slot = comm->mapped_count;
  }
  CUdeviceptr p = 0;
  const CUresult r =
      d.IpcOpenMemHandle(&p, handle, CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS);
  if (r != CUDA_SUCCESS)
    return comm_fail(cuda_message("mapping the root's output (IPC)", r));
  comm->mapped[slot] = {handle, p, comm->calls};
  ++comm->mapped_count;
  *base = p;
  return HEXIR_OK;
}

// Once, at set-up: the root exports its scratch buffer and every peer tries
// to map it.  Direct stores are used only if all of them could.
hexir_status_t probe_direct(hexir_comm_t *comm) {
  const Driver &d = driver();
  const Nccl &nc = nccl();
  CUstream s = comm->gather_stream;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(s);
  RootOutput *desc = &comm->desc_host[0];
  std::memset(desc, 0, sizeof(*desc));
  if (comm->rank == 0) {
    desc->magic = kRootOutputMagic;
    desc->valid = d.IpcGetMemHandle(&desc->handle, comm->scratch) == CUDA_SUCCESS;
    CUresult r = d.MemcpyHtoDAsync(comm->scratch, desc, sizeof(*desc), s);
    if (r != CUDA_SUCCESS)
      return comm_fail(cuda_message("probe descriptor", r));
  }
  void *buf = reinterpret_cast<void *>(comm->scratch);
  ncclResult_t nr = nc.Broadcast(buf, buf, kDescBytes, ncclUint8, 0, comm->comm, cs);
  if (nr != ncclSuccess)
    return comm_fail(nccl_message("ncclBroadcast (probe)", nr));
  CUresult r = d.MemcpyDtoHAsync(desc, comm->scratch, sizeof(*desc), s);
  if (r == CUDA_SUCCESS)
    r = d.StreamSynchronize(s);
  if (r != CUDA_SUCCESS)
    return comm_fail(cuda_message("probe descriptor", r));
  int32_t ok = desc->magic == kRootOutputMagic && desc->valid;
  if (ok && comm->rank != 0) {
    CUdeviceptr p = 0;
    ok = d.IpcOpenMemHandle(&p, desc->handle,
                            CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS) == CUDA_SUCCESS;
    if (ok)
      d.IpcCloseMemHandle(p);
  }
  const CUdeviceptr word = comm->scratch + kDescBytes;
  r = d.MemcpyHtoDAsync(word, &ok, sizeof(ok), s);
  if (r != CUDA_SUCCESS)
    return comm_fail(cuda_message("probe vote", r));
  void *w = reinterpret_cast<void *>(word);
  nr = nc.AllReduce(w, w, 1, ncclInt32, ncclMin, comm->comm, cs);
  if (nr != ncclSuccess)
    return comm_fail(nccl_message("ncclAllReduce (probe)", nr));
  r = d.MemcpyDtoHAsync(&ok, word, sizeof(ok), s);
  if (r == CUDA_SUCCESS)
    r = d.StreamSynchronize(s);
  if (r != CUDA_SUCCESS)
    return comm_fail(cuda_message("probe vote", r));
  comm->direct = ok == 1;
  return HEXIR_OK;
}

// The weight's k pieces for a broadcast that peers compute behind: a short
// first piece (512 of k) whose transfer is the only exposed one, then the
// rest, which lands long before the first piece's GEMM ends (8192 x 8192 on
// B200: the 480 MiB rest crosses NVLink in ~0.8 ms, the first piece takes
// ~2 ms of DMMA time on 8192 rows).  Each extra piece costs ~0.2 ms there
// (every CTA stores and reloads its partial sums, one more tail wave), so
// there are two.  Multiples of the 32-wide k tile.  One piece for a single
// rank (nothing to broadcast).  Returns the count.
constexpr uint32_t kBroadcastPieceMinK = 2048;
uint32_t broadcast_pieces(uint32_t k, uint32_t ranks, uint32_t bounds[3]) {
  bounds[0] = 0;
  if (ranks < 2 || k < kBroadcastPieceMinK) {
    bounds[1] = k;
    bounds[2] = k;
    return 1;
  }
  bounds[1] = 512;
  bounds[2] = k;
  return 2;
}

// Device workspace `*p` of at least `bytes` (kept between calls, grown as
// needed once the streams that used it are idle).
CUresult ensure_buffer(CUdeviceptr *p, size_t *have, size_t bytes) {
  if (*have >= bytes)
    return CUDA_SUCCESS;
  const Driver &d = driver();
  if (*p) {
    CUresult r = d.CtxSynchronize();
    if (r != CUDA_SUCCESS)
      return r;
    d.MemFree(*p);
    *p = 0;
    *have = 0;
  }
  CUresult r = d.MemAlloc(p, bytes ? bytes : 16);
  if (r == CUDA_SUCCESS)
    *have = bytes;
  return r;
}

CUdeviceptr failure_word(const hexir_comm_t *comm) {
  return comm->scratch + kDescBytes;
}

// Every rank, at the end of every sharded call, in the same order: a rank
// whose part failed marks the failure word, and a max all-reduce hands the
// mark to every rank on the caller's stream (where hexir_comm_synchronize
// reads it).  A rank that failed still takes this step, so no rank waits
// for ever on it.
hexir_status_t reduce_failure(hexir_comm_t *comm, CUstream s, bool failed) {
  const Driver &d = driver();
  CUresult r = CUDA_SUCCESS;
  if (failed)
    r = d.MemsetD32Async(failure_word(comm), 1u, 1, s);
  void *w = reinterpret_cast<void *>(failure_word(comm));
  const ncclResult_t nr = nccl().AllReduce(
      w, w, 1, ncclInt32, ncclMax, comm->comm, reinterpret_cast<cudaStream_t>(s));
  if (nr != ncclSuccess)
    return comm_fail(nccl_message("ncclAllReduce (failure word)", nr));
  if (r != CUDA_SUCCESS)
    return comm_fail(cuda_message("marking the failure word", r));
  return HEXIR_OK;
}

}  // namespace

namespace {
// Runs `fn` with a context current: the calling thread's own, when it has
// one (a process driving GPU r under torch or another runtime has GPU r's
// primary context current), else GPU 0's.  Page-locking is portable, so any
// context serves; borrowing GPU 0's where another GPU is in use would create
// a context on GPU 0 for nothing.
template <typename Fn>
hexir_status_t with_some_context(Fn fn) {
  const Driver &d = driver();
  if (!d.ok) {
    set_last_error(d.error);
    return HEXIR_ERROR_DEVICE;
  }
  CUcontext current = nullptr;
  if (d.CtxGetCurrent(&current) == CUDA_SUCCESS && current)
    return fn();
  std::string error;
  DeviceState *dev = device_state(0, &error);
  if (!dev) {
    set_last_error(error);
    return HEXIR_ERROR_DEVICE;
  }
  ContextGuard guard(dev->context);
  return fn();
}
}  // namespace

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

hexir_status_t hexir_shard_gather_pieces(uint64_t rows, uint32_t index,
                                         uint64_t *begin, uint64_t *count,
                                         uint32_t *pieces) {
  if (!begin || !count)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  if (!rows) {
    *begin = 0;
    *count = 0;
    if (pieces)
      *pieces = 0;
    return HEXIR_OK;
  }
  const uint32_t n = gather_piece(rows, index, begin, count);
  if (pieces)
    *pieces = n;
  return HEXIR_OK;
}

hexir_status_t hexir_shard_weight_pieces(uint32_t k, uint32_t ranks,
                                         uint32_t *bounds, uint32_t *pieces) {
  if (!bounds || !pieces || ranks == 0)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  uint32_t b[3];
  *pieces = broadcast_pieces(k, ranks, b);
  for (uint32_t i = 0; i <= *pieces; ++i)
    bounds[i] = b[i];
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
  // The side stream carries the weight pieces that peers' GEMMs wait for:
  // highest priority, so its NCCL kernels take SMs as soon as GEMM CTAs
  // retire instead of after the whole GEMM grid has been dispatched.
  int least = 0, greatest = 0;
  CUresult cr = d.CtxGetStreamPriorityRange(&least, &greatest);
  if (cr == CUDA_SUCCESS)
    cr = d.StreamCreateWithPriority(&comm->gather_stream, CU_STREAM_NON_BLOCKING,
                                    greatest);
  for (uint32_t i = 0; cr == CUDA_SUCCESS && i < kGatherChunks; ++i)
    cr = d.EventCreate(&comm->chunk_done[i], CU_EVENT_DISABLE_TIMING);
  if (cr == CUDA_SUCCESS)
    cr = d.EventCreate(&comm->gather_done, CU_EVENT_DISABLE_TIMING);
  for (uint32_t i = 0; cr == CUDA_SUCCESS && i < kDescSlots; ++i)
    cr = d.EventCreate(&comm->desc_done[i], CU_EVENT_DISABLE_TIMING);
  for (CUevent *ev : {&comm->w_start, &comm->w_piece[0], &comm->w_piece[1],
                      &comm->w_done, &comm->down_done})
    if (cr == CUDA_SUCCESS)
      cr = d.EventCreate(ev, CU_EVENT_DISABLE_TIMING);
  if (cr == CUDA_SUCCESS)
    cr = d.StreamCreate(&comm->up_stream, CU_STREAM_NON_BLOCKING);
  if (cr == CUDA_SUCCESS)
    cr = d.StreamCreate(&comm->down_stream, CU_STREAM_NON_BLOCKING);
  if (cr == CUDA_SUCCESS)
    cr = d.StreamCreate(&comm->side_stream, CU_STREAM_NON_BLOCKING);
  if (cr == CUDA_SUCCESS)
    cr = d.MemAlloc(&comm->scratch, kDescBytes + 16);
  if (cr == CUDA_SUCCESS)
    cr = d.MemAllocHost(reinterpret_cast<void **>(&comm->desc_host),
                        kDescSlots * sizeof(RootOutput));
  if (cr != CUDA_SUCCESS) {
    set_last_error(cuda_message("gather stream set-up", cr));
    hexir_comm_release(comm);
    return HEXIR_ERROR_DEVICE;
  }
  if (nranks > 1) {
    hexir_status_t st = probe_direct(comm);
    if (st != HEXIR_OK) {
      hexir_comm_release(comm);
      return st;
    }
  }
  // The probe used the failure word for its vote; no call has failed yet.
  cr = d.MemsetD32Async(failure_word(comm), 0u, 1, comm->gather_stream);
  if (cr == CUDA_SUCCESS)
    cr = d.StreamSynchronize(comm->gather_stream);
  if (cr != CUDA_SUCCESS) {
    set_last_error(cuda_message("clearing the failure word", cr));
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
    for (CUevent ev : {comm->w_start, comm->w_piece[0], comm->w_piece[1],
                       comm->w_done})
      if (ev)
        d.EventDestroy(ev);
    if (comm->mapped_count)
      d.CtxSynchronize();
    for (size_t i = 0; i < comm->mapped_count; ++i)
      d.IpcCloseMemHandle(comm->mapped[i].base);
    for (CUevent ev : comm->desc_done)
      if (ev) {
        d.EventSynchronize(ev);
        d.EventDestroy(ev);
      }
    if (comm->desc_host)
      d.MemFreeHost(comm->desc_host);
    if (comm->scratch)
      d.MemFree(comm->scratch);
    for (CUstream st : {comm->up_stream, comm->down_stream, comm->side_stream})
      if (st) {
        d.StreamSynchronize(st);
        d.StreamDestroy(st);
      }
    if (comm->down_done)
      d.EventDestroy(comm->down_done);
    for (CUdeviceptr p : {comm->a_dev, comm->w_dev, comm->c_dev})
      if (p)
        d.MemFree(p);
  }
  if (comm->comm && nccl().ok)
    nccl().CommDestroy(comm->comm);
  delete comm;
}

int hexir_comm_rank(const hexir_comm_t *comm) { return comm ? comm->rank : -1; }
int hexir_comm_size(const hexir_comm_t *comm) {
  return comm ? comm->nranks : 0;
}
int hexir_comm_direct_stores(const hexir_comm_t *comm) {
  return comm && comm->direct ? 1 : 0;
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
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(s);
  const Driver &d = driver();
  const uint32_t ranks = static_cast<uint32_t>(comm->nranks);
  uint64_t begin = 0, rows = 0;
  hexir_shard_rows(m, ranks, static_cast<uint32_t>(comm->rank), &begin, &rows);

  const bool root = comm->rank == 0;
  // The relu, and no stream-K: a rank's rows run in gather pieces, and its
  // block has the bits of one data-parallel or split-K launch.
  const uint32_t mm_flags = (flags & HEXIR_MATMUL_RELU) | HEXIR_MATMUL_NO_STREAM_K;
  const uint32_t my_rows = static_cast<uint32_t>(rows);
  // The weight goes out in k pieces (one for short k or a single rank).  A
  // rank computes behind them -- one launch per piece, each continuing the
  // previous one's sums, the same operations as one unsplit launch -- where
  // its one-shot plan has no k split; otherwise it runs that plan once the
  // whole weight has landed.
  uint32_t bounds[3] = {0, k, k};
  const uint32_t pieces = broadcast_pieces(k, ranks, bounds);
  const MatmulPlan one = plan_matmul(dev, a_rows, w, c, my_rows, n, k, mm_flags);
  const bool chain = pieces > 1 && one.split_k == 1 && !one.stream_k();

  // 0. Where the rows go: the root describes its c (IPC handle + offset)
  //    every call and every rank reads that description, so all of them
  //    take the same branch.  A peer reads it only after its first piece is
  //    queued, so the host round trip hides behind that piece.
  RootOutput *desc = nullptr;
  CUevent desc_ready = nullptr;
  bool direct = false;
  CUresult cr = CUDA_SUCCESS;
  if (ranks > 1 && comm->direct) {
    desc = next_desc(comm, &desc_ready);
    std::memset(desc, 0, sizeof(*desc));
    if (root) {
      CUdeviceptr base = 0;
      size_t size = 0;
      const CUdeviceptr cp = reinterpret_cast<CUdeviceptr>(c);
      desc->magic = kRootOutputMagic;
      desc->valid = !(flags & HEXIR_SHARD_GATHER_NCCL) &&
                    d.MemGetAddressRange(&base, &size, cp) == CUDA_SUCCESS &&
                    d.IpcGetMemHandle(&desc->handle, base) == CUDA_SUCCESS;
      desc->offset = desc->valid ? cp - base : 0;
      direct = desc->valid;
      cr = d.MemcpyHtoDAsync(comm->scratch, desc, sizeof(*desc), s);
    }
    if (cr != CUDA_SUCCESS)
      return comm_fail(cuda_message("output descriptor", cr));
    void *buf = reinterpret_cast<void *>(comm->scratch);
    ncclResult_t nr =
        nc.Broadcast(buf, buf, kDescBytes, ncclUint8, 0, comm->comm, cs);
    if (nr != ncclSuccess)
      return comm_fail(nccl_message("ncclBroadcast (output descriptor)", nr));
    if (!root)
      cr = d.MemcpyDtoHAsync(desc, comm->scratch, sizeof(*desc), s);
    if (cr == CUDA_SUCCESS)
      cr = d.EventRecord(desc_ready, s);
    if (cr != CUDA_SUCCESS)
      return comm_fail(cuda_message("output descriptor", cr));
  }

  // 1. The weight from the root to everyone over NVLink, piece by piece, on
  //    the high-priority side stream (it starts after the caller's queued
  //    work, which may have written w).
  CUstream bs = comm->gather_stream;
  cudaStream_t bcs = reinterpret_cast<cudaStream_t>(bs);
  cr = d.EventRecord(comm->w_start, s);
  if (cr == CUDA_SUCCESS)
    cr = d.StreamWaitEvent(bs, comm->w_start, 0);
  if (cr != CUDA_SUCCESS)
    return comm_fail(cuda_message("broadcast stream", cr));
  for (uint32_t j = 0; j < pieces; ++j) {
    double *wp = w + static_cast<size_t>(bounds[j]) * n;
    ncclResult_t nr =
        nc.Broadcast(wp, wp, static_cast<size_t>(bounds[j + 1] - bounds[j]) * n,
                     ncclDouble, 0, comm->comm, bcs);
    if (nr != ncclSuccess)
      return comm_fail(nccl_message("ncclBroadcast (weight)", nr));
    d.EventRecord(comm->w_piece[j], bs);
  }
  d.EventRecord(comm->w_done, bs);

  // 2. The first piece over all of this rank's rows (the root needs no
  //    broadcast): partial sums in c (a peer's staging rows).
  hexir_status_t status = HEXIR_OK;
  if (chain && my_rows) {
    if (!root)
      d.StreamWaitEvent(s, comm->w_piece[0], 0);
    status = launch_matmul(dev, lib, a_rows, w, c, my_rows, n, bounds[1],
                           HEXIR_MATMUL_SPLIT_K(1), s, &error, k, nullptr);
  }

  // 3. A peer learns where its rows go.
  CUdeviceptr remote_c = 0;
  if (desc && !root) {
    cr = d.EventSynchronize(desc_ready);
    if (cr != CUDA_SUCCESS)
      return comm_fail(cuda_message("output descriptor", cr));
    direct = desc->magic == kRootOutputMagic && desc->valid;
    if (direct && status == HEXIR_OK) {
      status = map_root_output(comm, desc->handle, &remote_c);
      remote_c += desc->offset;
    }
  }

  // The rest of this rank's rows [cb, cb + count): the remaining k pieces
  // continuing the first one's sums, or the one-shot plan.
  auto finish_rows = [&](uint64_t cb, uint64_t count, double *out,
                         uint32_t out_flags) -> hexir_status_t {
    if (!count)
      return HEXIR_OK;
    const uint32_t mm = static_cast<uint32_t>(count);
    if (!chain) {
      if (!root)
        d.StreamWaitEvent(s, comm->w_done, 0);
      return launch_matmul(dev, lib, a_rows + cb * k, w, out, mm, n, k,
                           mm_flags | out_flags, s, &error);
    }
    hexir_status_t st = HEXIR_OK;
    for (uint32_t j = 1; j < pieces && st == HEXIR_OK; ++j) {
      const bool last = j + 1 == pieces;
      if (!root)
        d.StreamWaitEvent(s, comm->w_piece[j], 0);
      st = launch_matmul(dev, lib, a_rows + cb * k + bounds[j],
                         w + static_cast<size_t>(bounds[j]) * n,
                         last ? out : c + cb * n, mm, n, bounds[j + 1] - bounds[j],
                         (last ? mm_flags | out_flags : 0u) | HEXIR_MATMUL_SPLIT_K(1),
                         s, &error, k, c + cb * n);
    }
    return st;
  };

  if (direct) {
    // 4. Every rank's kernel stores its output tiles into the root's c over
    //    NVLink (system-scope fence before each CTA retires); the failure
    //    word's all-reduce then orders the root's stream after every peer's
    //    kernels.  A rank whose launch failed still takes every collective
    //    step, so no rank waits for ever.
    if (status == HEXIR_OK) {
      double *out = root ? c : reinterpret_cast<double *>(remote_c) + begin * n;
      status = finish_rows(0, my_rows, out, root ? 0u : HEXIR_MATMUL_REMOTE_OUTPUT);
    }
    if (status != HEXIR_OK)
      set_last_error(error.empty() ? hexir_status_string(status) : error);
    d.StreamWaitEvent(s, comm->w_done, 0);
    const hexir_status_t rs = reduce_failure(comm, s, status != HEXIR_OK);
    return status != HEXIR_OK ? status : rs;
  }
  // 4'. Rows by NCCL: this rank's rows in up to kGatherChunks pieces of
  //     shrinking size; the root writes straight into its part of c, and
  //     each finished piece of a peer goes to the root on the side stream
  //     while the next piece computes.  Every rank splits its rows by the
  //     same rule, so the root knows each peer's pieces.  After a failed
  //     launch the rank stops computing but still takes every send/receive
  //     step, so no rank waits for ever, and reports the failure.
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
    if (i < my_chunks && status == HEXIR_OK) {
      uint64_t cb = 0, cnt = 0;
      gather_piece(rows, i, &cb, &cnt);
      status = finish_rows(cb, cnt, c + cb * n, 0u);
    }
    if (ranks == 1)
      continue;
    d.EventRecord(comm->chunk_done[i], s);
    d.StreamWaitEvent(comm->gather_stream, comm->chunk_done[i], 0);
    nc.GroupStart();
    if (root) {
      for (uint32_t peer = 1; peer < ranks; ++peer) {
        uint64_t pb = 0, pr = 0;
        hexir_shard_rows(m, ranks, peer, &pb, &pr);
        uint64_t cb = 0, cnt = 0;
        if (!pr)
          continue;
        gather_piece(pr, i, &cb, &cnt);
        if (cnt)
          nc.Recv(c + (pb + cb) * n, cnt * n, ncclDouble, static_cast<int>(peer),
                  comm->comm, gs);
      }
    } else if (i < my_chunks) {
      uint64_t cb = 0, cnt = 0;
      gather_piece(rows, i, &cb, &cnt);
      if (cnt)
        nc.Send(c + cb * n, cnt * n, ncclDouble, 0, comm->comm, gs);
    }
    ncclResult_t nr = nc.GroupEnd();
    if (nr != ncclSuccess) {
      set_last_error(nccl_message("ncclGroupEnd (row gather)", nr));
      return HEXIR_ERROR_DEVICE;
    }
  }
  // The caller's stream completes only after the broadcast and the gather.
  d.EventRecord(comm->gather_done, comm->gather_stream);
  d.StreamWaitEvent(s, comm->gather_done, 0);
  if (status != HEXIR_OK)
    set_last_error(error.empty() ? hexir_status_string(status) : error);
  if (ranks > 1) {
    const hexir_status_t rs = reduce_failure(comm, s, status != HEXIR_OK);
    if (status == HEXIR_OK)
      status = rs;
  }
  return status;
}

hexir_status_t hexir_sharded_linear_host_f64(hexir_comm_t *comm,
                                             const double *a_rows,
                                             const double *w, double *c_rows,
                                             uint32_t m, uint32_t n, uint32_t k,
                                             uint32_t flags, void *stream) {
  if (!comm)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  const uint32_t ranks = static_cast<uint32_t>(comm->nranks);
  const uint32_t rank = static_cast<uint32_t>(comm->rank);
  const bool w_everywhere = (flags & HEXIR_SHARD_W_ON_ALL) != 0;
  uint64_t begin = 0, rows = 0;
  hexir_shard_rows(m, ranks, rank, &begin, &rows);
  // Argument errors are the caller's on every rank alike (same m, n, k,
  // flags), so returning before any collective leaves no rank waiting.
  if ((rows && (!a_rows || !c_rows)) ||
      ((rank == 0 || w_everywhere) && !w && k && n))
    return HEXIR_ERROR_INVALID_ARGUMENT;
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
  const Driver &d = driver();
  const Nccl &nc = nccl();
  CUstream s = static_cast<CUstream>(stream);
  CUstream up = comm->up_stream, down = comm->down_stream;
  CUstream gs = comm->gather_stream;
  const size_t row_a = static_cast<size_t>(k) * 8, row_c = static_cast<size_t>(n) * 8;
  const size_t w_size = static_cast<size_t>(k) * row_c;
  // The relu, and no stream-K: rows run in chunks, each with the bits of
  // the same rows in one data-parallel or split-K launch.
  const uint32_t mm_flags = (flags & HEXIR_MATMUL_RELU) | HEXIR_MATMUL_NO_STREAM_K;

  bool failed = false;
  auto note = [&](CUresult r, const char *what) {
    if (r != CUDA_SUCCESS && !failed) {
      failed = true;
      error = cuda_message(what, r);
    }
    return r == CUDA_SUCCESS;
  };
  // 0. Workspace, agreed on: the weight gather below needs a buffer on
  //    every rank, so every rank learns whether any rank could not get its
  //    own (one word max-reduced and read back) and all return together.
  note(ensure_buffer(&comm->a_dev, &comm->a_bytes, rows * row_a), "cuMemAlloc (rows of a)");
  if (!failed)
    note(ensure_buffer(&comm->w_dev, &comm->w_bytes, w_size), "cuMemAlloc (weight)");
  if (!failed)
    note(ensure_buffer(&comm->c_dev, &comm->c_bytes, rows * row_c), "cuMemAlloc (rows of c)");
  if (ranks > 1) {
    hexir_status_t st = reduce_failure(comm, s, failed);
    if (st == HEXIR_OK)
      st = hexir_comm_synchronize(comm, stream);
    if (failed || st != HEXIR_OK) {
      if (failed)
        set_last_error(error);
      return failed ? HEXIR_ERROR_OUT_OF_MEMORY : st;
    }
  } else if (failed) {
    set_last_error(error);
    return HEXIR_ERROR_OUT_OF_MEMORY;
  }
  // From here a failure skips this rank's own work but still takes every
  // collective step: the weight gather and the failure word's reduction.

  // 1. The weight, in k pieces: every rank holding it uploads its own share
  //    of each piece's rows over its own host link and the shares meet over
  //    NVLink (one broadcast per share, grouped: an all-gather of unequal
  //    shares); otherwise the root uploads each piece and broadcasts it.
  //    For k >= 2048 the first half of k goes in growing pieces
  //    (weight_stream_bounds) so the GEMM starts after the first one, then
  //    the second half in one piece; every rank takes the same pieces (they
  //    depend on k alone).  Each copy starts after the caller's queued work
  //    (which may still read the workspace a previous call left).
  std::vector<uint32_t> bounds{0};
  uint32_t k1 = k;  // the streamed first half of k ends here
  if (k >= kBroadcastPieceMinK) {
    k1 = (k / 2) / 32 * 32;
    bounds = weight_stream_bounds(k1);
  }
  if (bounds.back() != k)
    bounds.push_back(k);
  const size_t pieces = bounds.size() - 1;
  const bool uploads_w = w_everywhere || rank == 0;
  CUevent start = comm->w_start;
  if (!failed)
    note(d.EventRecord(start, s), "cuEventRecord");
  if (!failed)
    note(d.StreamWaitEvent(up, start, 0), "cuStreamWaitEvent");
  if (!failed)
    note(d.StreamWaitEvent(down, start, 0), "cuStreamWaitEvent");
  if (!failed)
    note(d.StreamWaitEvent(gs, start, 0), "cuStreamWaitEvent");
  // Events of this call: the weight share of piece j uploaded (w_up) and
  // gathered (w_in), piece j's column band of a uploaded (band), each row
  // chunk's upload; destroyed once the caller's stream has passed them.
  std::vector<CUevent> events;
  auto event_on = [&](CUstream st) -> CUevent {
    CUevent ev = nullptr;
    if (!failed && note(d.EventCreate(&ev, CU_EVENT_DISABLE_TIMING), "cuEventCreate")) {
      events.push_back(ev);
      note(d.EventRecord(ev, st), "cuEventRecord");
    }
    return ev;
  };
  auto wait_on = [&](CUstream st, CUevent ev) {
    if (!failed && ev)
      note(d.StreamWaitEvent(st, ev, 0), "cuStreamWaitEvent");
  };

  // A rank continues its sums piece by piece over all its rows where its
  // one-shot plan has no k split (the same operations as one launch);
  // otherwise it runs that plan per row chunk once the whole weight is in.
  const MatmulPlan plan = plan_matmul(
      dev, reinterpret_cast<const double *>(comm->a_dev),
      reinterpret_cast<const double *>(comm->w_dev),
      reinterpret_cast<const double *>(comm->c_dev), static_cast<uint32_t>(rows),
      n, k, mm_flags);
  const bool chain = pieces > 1 && plan.split_k == 1 && !plan.stream_k() && rows;
  const uint32_t chunk_flags = mm_flags | HEXIR_MATMUL_SPLIT_K(plan.split_k);

  // a's columns [c0, c1) of rows [r0, r0 + nr), a 2-D copy (row pitch k).
  auto upload_band = [&](uint64_t r0, uint64_t nr, uint32_t c0, uint32_t c1) {
    if (failed || !nr || c1 <= c0)
      return;
    CUDA_MEMCPY2D cp;
    std::memset(&cp, 0, sizeof(cp));
    cp.srcMemoryType = CU_MEMORYTYPE_HOST;
    cp.srcHost = a_rows + r0 * k + c0;
    cp.srcPitch = row_a;
    cp.dstMemoryType = CU_MEMORYTYPE_DEVICE;
    cp.dstDevice = comm->a_dev + r0 * row_a + static_cast<size_t>(c0) * 8;
    cp.dstPitch = row_a;
    cp.WidthInBytes = static_cast<size_t>(c1 - c0) * 8;
    cp.Height = nr;
    note(d.Memcpy2DAsync(&cp, up), "row upload");
  };

  std::vector<CUevent> w_in(pieces, nullptr), band(pieces, nullptr);
  cudaStream_t g = reinterpret_cast<cudaStream_t>(gs);
  for (size_t j = 0; j < pieces; ++j) {
    const uint32_t p0 = bounds[j], p1 = bounds[j + 1];
    uint64_t sb = 0, sc = p1 - p0;
    if (w_everywhere)
      hexir_shard_rows(p1 - p0, ranks, rank, &sb, &sc);
    if (!failed && uploads_w && sc)
      note(d.MemcpyHtoDAsync(comm->w_dev + (p0 + sb) * row_c, w + (p0 + sb) * n,
                             sc * row_c, up),
           "weight upload");
    wait_on(gs, event_on(up));
    if (ranks > 1) {
      // Posted whatever happened above: every rank takes every step.
      ncclResult_t nr = ncclSuccess;
      if (w_everywhere) {
        nc.GroupStart();
        for (uint32_t r = 0; r < ranks; ++r) {
          uint64_t rb = 0, rc = 0;
          hexir_shard_rows(p1 - p0, ranks, r, &rb, &rc);
          if (!rc)
            continue;
          void *share = reinterpret_cast<void *>(comm->w_dev + (p0 + rb) * row_c);
          nc.Broadcast(share, share, rc * n, ncclDouble, static_cast<int>(r),
                       comm->comm, g);
        }
        nr = nc.GroupEnd();
      } else {
        void *piece = reinterpret_cast<void *>(comm->w_dev + static_cast<size_t>(p0) * row_c);
        nr = nc.Broadcast(piece, piece, static_cast<size_t>(p1 - p0) * n,
                          ncclDouble, 0, comm->comm, g);
      }
      if (nr != ncclSuccess && !failed) {
        failed = true;
        error = nccl_message("weight gather", nr);
      }
    }
    w_in[j] = event_on(gs);
    // The rows' columns of this piece, for a rank that computes behind it
    // (the last piece's columns go with the row chunks below).
    if (chain && j + 1 < pieces) {
      upload_band(0, rows, p0, p1);
      band[j] = event_on(up);
    }
  }

  // 2. Compute.  Phase 1 (chain): each piece of the first half over all
  //    the rank's rows, continuing the previous piece's sums in c.  Phase 2:
  //    per row chunk, the rest of k (or all of it), the relu, and the chunk's
  //    download into c_rows while the next chunk computes.
  hexir_status_t st = HEXIR_OK;
  if (chain) {
    for (size_t j = 0; j + 1 < pieces && !failed; ++j) {
      wait_on(s, w_in[j]);
      wait_on(s, band[j]);
      if (failed)
        break;
      st = launch_matmul(
          dev, lib, reinterpret_cast<const double *>(comm->a_dev + static_cast<size_t>(bounds[j]) * 8),
          reinterpret_cast<const double *>(comm->w_dev + static_cast<size_t>(bounds[j]) * row_c),
          reinterpret_cast<double *>(comm->c_dev), static_cast<uint32_t>(rows), n,
          bounds[j + 1] - bounds[j], HEXIR_MATMUL_SPLIT_K(1), s, &error, k,
          j ? reinterpret_cast<const double *>(comm->c_dev) : nullptr);
      if (st != HEXIR_OK)
        failed = true;
    }
  } else {
    for (size_t j = 0; j < pieces; ++j)
      wait_on(s, w_in[j]);
  }
  if (chain)
    wait_on(s, w_in[pieces - 1]);
  // The row chunks are independent: odd ones run on the side stream, which
  // starts after everything queued on `s` so far, so each chunk's last wave
  // of tiles overlaps the next one's first; `s` joins it after the chunks.
  CUstream side = comm->side_stream;
  wait_on(side, event_on(s));
  for (uint32_t i = 0; i < kHostChunks && !failed; ++i) {
    uint64_t cb = 0, cnt = 0;
    host_chunk(rows, i, &cb, &cnt);
    if (!cnt)
      continue;
    const CUstream on = i % 2 ? side : s;
    if (chain)
      upload_band(cb, cnt, bounds[pieces - 1], k);
    else if (!failed)
      note(d.MemcpyHtoDAsync(comm->a_dev + cb * row_a, a_rows + cb * k,
                             cnt * row_a, up),
           "row upload");
    wait_on(on, event_on(up));
    if (failed)
      break;
    if (chain) {
      const uint32_t kl = bounds[pieces - 1];
      st = launch_matmul(
          dev, lib,
          reinterpret_cast<const double *>(comm->a_dev + cb * row_a + static_cast<size_t>(kl) * 8),
          reinterpret_cast<const double *>(comm->w_dev + static_cast<size_t>(kl) * row_c),
          reinterpret_cast<double *>(comm->c_dev + cb * row_c),
          static_cast<uint32_t>(cnt), n, k - kl, mm_flags | HEXIR_MATMUL_SPLIT_K(1), on,
          &error, k, reinterpret_cast<const double *>(comm->c_dev + cb * row_c));
    } else {
      st = launch_matmul(
          dev, lib, reinterpret_cast<const double *>(comm->a_dev + cb * row_a),
          reinterpret_cast<const double *>(comm->w_dev),
          reinterpret_cast<double *>(comm->c_dev + cb * row_c),
          static_cast<uint32_t>(cnt), n, k, chunk_flags, on, &error);
    }
    if (st != HEXIR_OK) {
      failed = true;
      break;
    }
    wait_on(down, event_on(on));
    if (!failed)
      note(d.MemcpyDtoHAsync(c_rows + cb * n, comm->c_dev + cb * row_c,
                             cnt * row_c, down),
           "row download");
  }
  // The caller's stream waits for everything this call queued elsewhere.
  wait_on(s, event_on(side));
  wait_on(s, event_on(gs));
  wait_on(s, event_on(up));
  // ... and its downloads.
  d.EventRecord(comm->down_done, down);
  d.StreamWaitEvent(s, comm->down_done, 0);
  if (failed)
    set_last_error(error.empty() ? "sharded linear (host buffers) failed" : error);
  hexir_status_t rs = HEXIR_OK;
  if (ranks > 1)
    rs = reduce_failure(comm, s, failed);
  // 3. Synchronous: the rows are in c_rows on return, and a failure on any
  //    rank is reported on every rank.
  hexir_status_t ss = hexir_comm_synchronize(comm, stream);
  if (ss != HEXIR_OK || failed) {
    // The caller's stream may not have joined the others: let everything
    // queued on them finish before the events go and the workspace is
    // reused.
    d.StreamSynchronize(up);
    d.StreamSynchronize(down);
    d.StreamSynchronize(gs);
    d.StreamSynchronize(side);
  }
  for (CUevent ev : events)
    d.EventDestroy(ev);
  if (failed)
    return HEXIR_ERROR_DEVICE;
  return rs != HEXIR_OK ? rs : ss;
}

hexir_status_t hexir_host_register(void *ptr, size_t bytes) {
  if (!ptr || !bytes)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  return with_some_context([&]() {
    const CUresult r =
        driver().MemHostRegister(ptr, bytes, CU_MEMHOSTREGISTER_PORTABLE);
    return r == CUDA_SUCCESS ? HEXIR_OK
                             : comm_fail(cuda_message("cuMemHostRegister", r));
  });
}

hexir_status_t hexir_host_unregister(void *ptr) {
  if (!ptr)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  return with_some_context([&]() {
    const CUresult r = driver().MemHostUnregister(ptr);
    return r == CUDA_SUCCESS ? HEXIR_OK
                             : comm_fail(cuda_message("cuMemHostUnregister", r));
  });
}

hexir_status_t hexir_comm_synchronize(hexir_comm_t *comm, void *stream) {
  if (!comm)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  std::string error;
  DeviceState *dev = device_state(comm->ordinal, &error);
  if (!dev) {
    set_last_error(error);
    return HEXIR_ERROR_DEVICE;
  }
  CUstream s = static_cast<CUstream>(stream);
  // The stream's work, and the error words of this GPU's kernels.
  hexir_status_t st = check_device(dev, s, &error);
  if (st != HEXIR_OK) {
    set_last_error(error);
    return st;
  }
  if (comm->nranks < 2)
    return HEXIR_OK;
  ContextGuard guard(dev->context);
  const Driver &d = driver();
  int32_t failed = 0;
  CUresult r = d.MemcpyDtoHAsync(&failed, failure_word(comm), sizeof(failed), s);
  if (r == CUDA_SUCCESS)
    r = d.StreamSynchronize(s);
  if (r == CUDA_SUCCESS && failed) {
    r = d.MemsetD32Async(failure_word(comm), 0u, 1, s);
    if (r == CUDA_SUCCESS)
      r = d.StreamSynchronize(s);
  }
  if (r != CUDA_SUCCESS)
    return comm_fail(cuda_message("reading the failure word", r));
  if (failed)
    return comm_fail("a rank's part of a sharded linear failed since the last "
                     "hexir_comm_synchronize (that rank's own call returned "
                     "the error); the root's output rows are not valid");
  return HEXIR_OK;
}

}  // extern "C"
