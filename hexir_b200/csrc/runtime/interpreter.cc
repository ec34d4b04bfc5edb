// interpreter.cc -- replay an entry point's command list (include/hexir_runtime/vm.h).
//
// Command semantics follow the reference interpreter
// (runtime/src/vm/interpreter.c:200-340): ALLOC binds a zeroed destination,
// CONST binds RODATA bytes, DISPATCH runs an executable with the destination
// last, PRINT prints "%f " per element and a newline per row, END captures
// the last dispatch destination and releases everything.  Every number read
// from the module (slot, executable index, RODATA range, operand count) is
// bounds checked before use, and so are buffer sizes against the kernel
// extents (the reference trusts those).
//
// What is new is where values live.  A slot can have a host copy (RODATA or
// a host buffer) and a copy on any open GPU; a dispatch makes its inputs
// valid where it runs (host<->device copies, or NVLink peer copies) and its
// destination valid only there.  That lets cpu- and cuda-placed kernels mix
// in one program, and lets a linear be row-sharded over several GPUs:
//
//   weight  -> first GPU, then ncclBroadcast to the rest of the range
//   a rows  -> each GPU gets its rows (hexir_shard_rows) straight from where
//              a lives
//   c rows  -> each GPU computes its rows with no collective and stores them
//              straight into c on the first GPU over NVLink (peer access);
//              without peer access, ncclSend/Recv gathers them instead

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <new>
#include <set>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include "cuda_driver.h"
#include "fault.h"
#include "hal_internal.h"
#include "hexir_b200/comm.h"
#include "hexir_b200/kernels.h"
#include "hexir_runtime/program.h"
#include "hexir_runtime/vm.h"
#include "kernel_lib.h"
#include "module_internal.h"
#include "nccl_shim.h"

namespace hexir {

namespace {

constexpr int kMaxSlots = 256;  // as the reference (interpreter.c:20)

thread_local double g_last_kernel_ms = 0.0;

// NCCL communicators for in-process row sharding, one set per group of CUDA
// ordinals; kept for the life of the process.
std::mutex g_comms_mu;
std::map<std::vector<int>, std::vector<ncclComm_t>> g_comms;

hexir_status_t comms_for(const std::vector<int> &ordinals,
                         std::vector<ncclComm_t> *out, std::string *error) {
  std::lock_guard<std::mutex> lock(g_comms_mu);
  auto it = g_comms.find(ordinals);
  if (it != g_comms.end()) {
    *out = it->second;
    return HEXIR_OK;
  }
  const Nccl &n = nccl();
  if (!n.ok) {
    *error = n.error;
    return HEXIR_ERROR_DEVICE;
  }
  std::vector<ncclComm_t> comms(ordinals.size());
  ncclResult_t r = n.CommInitAll(comms.data(), static_cast<int>(ordinals.size()),
                                 ordinals.data());
  if (r != ncclSuccess) {
    *error = nccl_message("ncclCommInitAll", r);
    return HEXIR_ERROR_DEVICE;
  }
  g_comms[ordinals] = comms;
  *out = comms;
  return HEXIR_OK;
}

// Page-locked RODATA, set up the first time a program copies a large
// constant to a GPU and kept until the module is released, so every upload
// runs at pinned-memory speed.  The module's bytes are registered in place
// when the driver accepts that (heap copies); a file mapping it refuses is
// copied once into pinned host memory.  Without either, uploads stay on the
// driver's pageable path.
struct PinnedRodata {
  const uint8_t *src = nullptr;  // RODATA in the module
  uint64_t size = 0;
  void *registered = nullptr;    // page-aligned base registered in place
  uint8_t *copy = nullptr;       // pinned copy of RODATA
};

PinnedRodata *pin_rodata(const hexir_module_t *module) {
  auto *pin = new (std::nothrow) PinnedRodata;
  if (!pin)
    return nullptr;
  const void *data = nullptr;
  uint64_t size = 0;
  const Driver &d = driver();
  if (!d.ok ||
      hexir_module_section(module, HEXIR_SECTION_RODATA, &data, &size) != HEXIR_OK)
    return pin;
  pin->src = static_cast<const uint8_t *>(data);
  pin->size = size;
  const uintptr_t page = 4096;
  const uintptr_t begin = reinterpret_cast<uintptr_t>(data) & ~(page - 1);
  const uintptr_t end =
      (reinterpret_cast<uintptr_t>(data) + size + page - 1) & ~(page - 1);
  if (d.MemHostRegister(reinterpret_cast<void *>(begin), end - begin,
                        CU_MEMHOSTREGISTER_PORTABLE |
                            CU_MEMHOSTREGISTER_READ_ONLY) == CUDA_SUCCESS) {
    pin->registered = reinterpret_cast<void *>(begin);
    return pin;
  }
  void *host = nullptr;
  if (d.MemAllocHost(&host, size) == CUDA_SUCCESS) {
    std::memcpy(host, data, size);
    pin->copy = static_cast<uint8_t *>(host);
  }
  return pin;
}

void unpin_rodata(PinnedRodata *pin) {
  if (pin->registered)
    driver().MemHostUnregister(pin->registered);
  if (pin->copy)
    driver().MemFreeHost(pin->copy);
  delete pin;
}

// A constant kept on one GPU between executes of its module.
struct ResidentConst {
  DeviceState *device = nullptr;
  uint64_t offset = 0, bytes = 0;  // range of RODATA
  CUdeviceptr ptr = 0;
  CUevent ready = nullptr;  // the upload, recorded on the uploading stream
};

// Runtime state attached to a loaded module for its lifetime: the pinned
// RODATA (set up by the first large upload) and, when the caller asked for
// it (hexir_module_keep_constants), device copies of its constants.
struct ModuleState {
  const hexir_module_t *module = nullptr;
  std::once_flag pin_once;
  PinnedRodata *pin = nullptr;
  std::atomic<bool> keep_constants{false};
  std::mutex mu;  // guards resident
  std::vector<ResidentConst> resident;

  PinnedRodata *pinned() {
    std::call_once(pin_once, [this] { pin = pin_rodata(module); });
    return pin;
  }

  // Frees every resident copy once the GPU has finished using it.  Callers
  // hold mu.
  void drop_resident() {
    const Driver &d = driver();
    for (ResidentConst &rc : resident) {
      ContextGuard guard(rc.device->context);
      d.CtxSynchronize();
      if (rc.ready)
        d.EventDestroy(rc.ready);
      d.MemFree(rc.ptr);
    }
    resident.clear();
  }
};

void *make_module_state(const hexir_module_t *module) {
  auto *ms = new (std::nothrow) ModuleState;
  if (ms)
    ms->module = module;
  return ms;
}

void free_module_state(void *p) {
  auto *ms = static_cast<ModuleState *>(p);
  {
    std::lock_guard<std::mutex> lock(ms->mu);
    ms->drop_resident();
  }
  if (ms->pin)
    unpin_rodata(ms->pin);
  delete ms;
}

ModuleState *module_state(const hexir_module_t *module) {
  return module ? static_cast<ModuleState *>(module_attached(
                      module, make_module_state, free_module_state))
                : nullptr;
}

struct Slot {
  bool defined = false;
  uint64_t bytes = 0;
  const uint8_t *rodata = nullptr;  // CONST: bytes in the module mapping
  // Host copy: a page-locked block the Vm owns (when the execute has GPUs)
  // or host_own's storage; never zero-filled unless the slot is zero.
  double *host = nullptr;
  std::unique_ptr<double[]> host_own;
  bool host_valid = false;
  bool zero = false;                // ALLOC'd and not written yet
  std::map<int, hexir_buffer_t *> dev;  // program ordinal -> buffer
  std::set<int> dev_valid;
};

struct Span {
  CudaDevice *device = nullptr;
  CUevent start = nullptr, stop = nullptr;
};

struct Vm {
  const hexir_module_t *module = nullptr;
  const uint8_t *rodata = nullptr;
  uint64_t rodata_size = 0;
  const hexir_executable_entry_t *exes = nullptr;
  uint32_t exe_count = 0;
  const uint8_t *exe_base = nullptr;
  uint64_t exe_size = 0;
  const hexir_launch_entry_t *launches = nullptr;
  uint32_t launch_count = 0;

  hexir_device_t *primary = nullptr;  // device named in messages
  std::vector<CudaDevice *> cuda;     // program ordinal -> device
  std::map<std::pair<uint32_t, int>, KernelLib *> libs;
  Slot slots[kMaxSlots];
  std::vector<std::pair<CudaDevice *, hexir_buffer_t *>> temps;
  std::vector<Span> spans;
  // Page-locked host blocks of this execute: they go back to the process
  // pool at release, after settle() has drained every stream that could
  // still copy from them (a pinned host-to-device copy is asynchronous).
  std::vector<std::pair<void *, size_t>> pinned;
  // Constants uploaded ahead of the dispatch that reads them, by (RODATA
  // offset, program ordinal): the buffer and the event its upload records
  // on the device's copy stream.  A CONST that binds the offset adopts the
  // buffer (see prefetch_ahead).
  struct Prefetched {
    uint64_t bytes = 0;
    hexir_buffer_t *buffer = nullptr;
    CUevent ready = nullptr;
  };
  std::map<std::pair<uint64_t, int>, Prefetched> prefetched;
  uint64_t prefetched_bytes = 0;
  const uint8_t *program = nullptr;
  uint64_t program_size = 0;
  bool trace = false;

  // Capture target of hexir_execute_capture and the program offset of the
  // entry's last DISPATCH, whose destination is what gets captured: a large
  // last dispatch copies its rows out as they finish (see run_pipelined).
  void *capture_out = nullptr;
  size_t capture_size = 0;
  // A capture buffer that is not page-locked: results land in a pooled
  // page-locked block (capture_out) and reach the caller's memory
  // (capture_user) by host-thread copies, chunk by chunk as each finished
  // chunk's download completes (staged_chunks: offset, bytes, event).
  void *capture_user = nullptr;
  std::vector<std::tuple<uint64_t, uint64_t, CUevent>> staged_chunks;
  size_t staged_copied = 0;
  uint64_t last_dispatch_pc = UINT64_MAX;
  uint64_t current_pc = 0;
  bool capture_done = false;

  ~Vm() { release(); }

  void release() {
    for (Slot &s : slots) {
      for (auto &kv : s.dev)
        hexir_buffer_release(kv.second);
      s = Slot();
    }
    for (auto &t : temps)
      hexir_buffer_release(t.second);
    temps.clear();
    for (auto &chunk : staged_chunks) {
      ContextGuard guard(cuda.front()->state->context);
      driver().EventSynchronize(std::get<2>(chunk));
      driver().EventDestroy(std::get<2>(chunk));
    }
    staged_chunks.clear();
    for (auto &b : pinned)
      pinned_give(b.first, b.second);
    pinned.clear();
    for (auto &kv : prefetched) {
      CudaDevice *dev = cuda[kv.first.second];
      ContextGuard guard(dev->state->context);
      // An upload nobody adopted (an execute that failed first).
      driver().EventSynchronize(kv.second.ready);
      driver().EventDestroy(kv.second.ready);
      hexir_buffer_release(kv.second.buffer);
    }
    prefetched.clear();
    prefetched_bytes = 0;
    for (Span &sp : spans) {
      ContextGuard guard(sp.device->state->context);
      driver().EventDestroy(sp.start);
      driver().EventDestroy(sp.stop);
    }
    spans.clear();
  }

  Slot *slot(uint64_t index) {
    return index < kMaxSlots && slots[index].defined ? &slots[index] : nullptr;
  }

  // ---- binding -----------------------------------------------------------

  hexir_status_t bind(uint64_t index, uint64_t bytes) {
    // A slot larger than any memory (1 TiB) is a malformed module; the cap
    // also keeps every size computation below from wrapping.
    constexpr uint64_t kMaxSlotBytes = 1ull << 40;
    if (index >= kMaxSlots || bytes > kMaxSlotBytes)
      return HEXIR_ERROR_INVALID_MODULE;
    Slot &s = slots[index];
    for (auto &kv : s.dev)
      hexir_buffer_release(kv.second);
    s = Slot();
    s.defined = true;
    s.bytes = bytes;
    return HEXIR_OK;
  }

  // ---- where values live -------------------------------------------------

  // Order `to`'s stream after the work queued so far on `from`'s stream.
  hexir_status_t order_after(CudaDevice *from, CudaDevice *to) {
    if (from == to)
      return HEXIR_OK;
    const Driver &d = driver();
    CUevent ev = nullptr;
    ContextGuard g(from->state->context);
    CUresult r = d.EventCreate(&ev, CU_EVENT_DISABLE_TIMING);
    if (r == CUDA_SUCCESS)
      r = d.EventRecord(ev, from->stream);
    if (r == CUDA_SUCCESS) {
      ContextGuard g2(to->state->context);
      r = d.StreamWaitEvent(to->stream, ev, 0);
    }
    if (ev)
      d.EventDestroy(ev);  // deferred by the driver until the event completes
    if (r != CUDA_SUCCESS) {
      report(cuda_message("cross-device ordering", r));
      return HEXIR_ERROR_DEVICE;
    }
    return HEXIR_OK;
  }

  // Whether `from` may load and store `to`'s memory directly (NVLink peer
  // access), enabling it on first use.
  static bool peer_access(CudaDevice *from, CudaDevice *to) {
    static std::mutex mu;
    static std::map<std::pair<CUcontext, CUcontext>, bool> known;
    if (from->state == to->state)
      return true;
    const auto key = std::make_pair(from->state->context, to->state->context);
    std::lock_guard<std::mutex> lock(mu);
    auto it = known.find(key);
    if (it != known.end())
      return it->second;
    const Driver &d = driver();
    int can = 0;
    bool ok = d.DeviceCanAccessPeer(&can, from->state->device,
                                    to->state->device) == CUDA_SUCCESS &&
              can;
    if (ok) {
      ContextGuard guard(from->state->context);
      const CUresult r = d.CtxEnablePeerAccess(to->state->context, 0);
      ok = r == CUDA_SUCCESS || r == CUDA_ERROR_PEER_ACCESS_ALREADY_ENABLED;
    }
    known[key] = ok;
    return ok;
  }

  hexir_status_t buffer_on(Slot &s, int o, uint64_t bytes, CUdeviceptr *out) {
    auto it = s.dev.find(o);
    if (it == s.dev.end()) {
      hexir_buffer_t *b = nullptr;
      hexir_status_t st = cuda[o]->allocate_pooled(bytes, &b);
      if (st != HEXIR_OK)
        return st;
      it = s.dev.emplace(o, b).first;
    }
    *out = reinterpret_cast<CUdeviceptr>(it->second->impl);
    return HEXIR_OK;
  }

  hexir_status_t temp_on(int o, uint64_t bytes, CUdeviceptr *out) {
    hexir_buffer_t *b = nullptr;
    hexir_status_t st = cuda[o]->allocate_pooled(bytes, &b);
    if (st != HEXIR_OK)
      return st;
    temps.emplace_back(cuda[o], b);
    *out = reinterpret_cast<CUdeviceptr>(b->impl);
    return HEXIR_OK;
  }

  // Where to upload RODATA bytes from: the pinned copy of RODATA when the
  // module has one (large uploads set it up), else the module's own bytes.
  const uint8_t *rodata_source(const Slot &s, uint64_t offset, uint64_t bytes) {
    const uint8_t *src = s.rodata + offset;
    ModuleState *ms = bytes >= (1u << 20) ? module_state(module) : nullptr;
    if (ms) {
      PinnedRodata *pin = ms->pinned();
      if (pin && pin->copy && src >= pin->src && src + bytes <= pin->src + pin->size)
        src = pin->copy + (src - pin->src);
    }
    return src;
  }

  // Copy bytes [offset, offset + bytes) of slot s to `dst` on GPU o, from
  // wherever the slot is valid.  Asynchronous on o's stream.
  hexir_status_t copy_range_to(Slot &s, uint64_t offset, uint64_t bytes, int o,
                               CUdeviceptr dst) {
    const Driver &d = driver();
    CudaDevice *to = cuda[o];
    if (bytes == 0)
      return HEXIR_OK;
    ContextGuard guard(to->state->context);
    CUresult r = CUDA_SUCCESS;
    if (s.zero) {
      r = d.MemsetD8Async(dst, 0, bytes, to->stream);
    } else if (s.rodata) {
      return to->write_async(dst, rodata_source(s, offset, bytes), bytes);
    } else if (s.host_valid) {
      return to->write_async(
          dst, reinterpret_cast<const uint8_t *>(s.host) + offset, bytes);
    } else if (s.dev_valid.count(o)) {
      r = d.MemcpyDtoDAsync(
          dst, reinterpret_cast<CUdeviceptr>(s.dev[o]->impl) + offset, bytes,
          to->stream);
    } else if (!s.dev_valid.empty()) {
      const int p = *s.dev_valid.begin();
      CudaDevice *from = cuda[p];
      hexir_status_t st = order_after(from, to);
      if (st != HEXIR_OK)
        return st;
      r = d.MemcpyPeerAsync(dst, to->state->context,
                            reinterpret_cast<CUdeviceptr>(s.dev[p]->impl) +
                                offset,
                            from->state->context, bytes, to->stream);
      // Later work on `from` must not overwrite the source under the copy.
      if (r == CUDA_SUCCESS && (st = order_after(to, from)) != HEXIR_OK)
        return st;
    } else {
      r = d.MemsetD8Async(dst, 0, bytes, to->stream);
    }
    if (r != CUDA_SUCCESS) {
      report(cuda_message("device copy", r));
      return HEXIR_ERROR_DEVICE;
    }
    return HEXIR_OK;
  }

  // Attach the resident copy of constant slot s on GPU o, uploading it on
  // first use, when the module keeps its constants.  *done is false when the
  // slot is not served that way (the caller uploads as usual).
  hexir_status_t resident_on(Slot &s, int o, CUdeviceptr *out, bool *done) {
    *done = false;
    ModuleState *ms = s.rodata && s.bytes ? module_state(module) : nullptr;
    if (!ms || !ms->keep_constants.load() || s.dev.count(o))
      return HEXIR_OK;
    CudaDevice *dev = cuda[o];
    const Driver &d = driver();
    const uint64_t offset = static_cast<uint64_t>(s.rodata - rodata);
    std::lock_guard<std::mutex> lock(ms->mu);
    ContextGuard guard(dev->state->context);
    ResidentConst *rc = nullptr;
    for (ResidentConst &r : ms->resident)
      if (r.device == dev->state && r.offset == offset && r.bytes == s.bytes)
        rc = &r;
    auto *b = new (std::nothrow) hexir_buffer_t;
    if (!b)
      return HEXIR_ERROR_OUT_OF_MEMORY;
    if (!rc) {
      ResidentConst fresh;
      fresh.device = dev->state;
      fresh.offset = offset;
      fresh.bytes = s.bytes;
      if (fault_hit(FaultSite::Alloc) ||
          d.MemAlloc(&fresh.ptr, s.bytes) != CUDA_SUCCESS) {
        delete b;  // no room to keep it: upload per execute as usual
        return HEXIR_OK;
      }
      hexir_status_t st = dev->write_async(fresh.ptr, rodata_source(s, 0, s.bytes),
                                           s.bytes);
      CUresult r = st == HEXIR_OK
                       ? d.EventCreate(&fresh.ready, CU_EVENT_DISABLE_TIMING)
                       : CUDA_SUCCESS;
      if (st == HEXIR_OK && r == CUDA_SUCCESS)
        r = d.EventRecord(fresh.ready, dev->stream);
      if (st != HEXIR_OK || r != CUDA_SUCCESS) {
        d.StreamSynchronize(dev->stream);
        if (fresh.ready)
          d.EventDestroy(fresh.ready);
        d.MemFree(fresh.ptr);
        delete b;
        if (st == HEXIR_OK)
          report(cuda_message("resident constant upload", r));
        return st == HEXIR_OK ? HEXIR_ERROR_DEVICE : st;
      }
      ms->resident.push_back(fresh);
      rc = &ms->resident.back();
    } else if (d.StreamWaitEvent(dev->stream, rc->ready, 0) != CUDA_SUCCESS) {
      delete b;
      return HEXIR_ERROR_DEVICE;
    }
    b->device = dev;
    b->size = s.bytes;
    b->memory = HEXIR_MEMORY_DEVICE_LOCAL;
    b->impl = reinterpret_cast<void *>(rc->ptr);
    b->borrowed = true;
    s.dev[o] = b;
    s.dev_valid.insert(o);
    *out = rc->ptr;
    *done = true;
    return HEXIR_OK;
  }

  // Resident copies are shared by every execute: a slot that is about to be
  // written lets go of them first (they stay with the module).
  static void drop_borrowed(Slot &s) {
    for (auto it = s.dev.begin(); it != s.dev.end();) {
      if (it->second->borrowed) {
        s.dev_valid.erase(it->first);
        delete it->second;
        it = s.dev.erase(it);
      } else {
        ++it;
      }
    }
  }

  // A buffer of slot s on GPU o that may be written.
  hexir_status_t writable_on(Slot &s, int o, uint64_t bytes, CUdeviceptr *out) {
    auto it = s.dev.find(o);
    if (it != s.dev.end() && it->second->borrowed) {
      s.dev_valid.erase(o);
      delete it->second;
      s.dev.erase(it);
    }
    return buffer_on(s, o, bytes, out);
  }

  // Make slot s valid on GPU o and return its address there.
  hexir_status_t on_device(Slot &s, int o, CUdeviceptr *out) {
    bool resident = false;
    hexir_status_t st = resident_on(s, o, out, &resident);
    if (st != HEXIR_OK || resident)
      return st;
    st = buffer_on(s, o, s.bytes, out);
    if (st != HEXIR_OK || s.dev_valid.count(o))
      return st;
    st = copy_range_to(s, 0, s.bytes, o, *out);
    if (st == HEXIR_OK)
      s.dev_valid.insert(o);
    return st;
  }

  // Make slot s valid on the host and return its bytes.
  hexir_status_t on_host(Slot &s, const uint8_t **out) {
    if (s.rodata && (reinterpret_cast<uintptr_t>(s.rodata) & 7u) == 0) {
      *out = s.rodata;
      return HEXIR_OK;
    }
    if (!s.host_valid && fault_hit(FaultSite::Alloc))
      return HEXIR_ERROR_OUT_OF_MEMORY;
    if (s.rodata && !s.host_valid) {
      // A CONST at an offset that is not a multiple of 8 (the serializer
      // never writes one): the host kernels read an aligned copy.
      double *h = host_storage(s);
      std::memcpy(h, s.rodata, static_cast<size_t>(s.bytes));
      s.host_valid = true;
    }
    if (!s.host_valid) {
      double *h = host_storage(s);
      if (!s.zero && !s.dev_valid.empty()) {
        // Every byte comes from the device copy.
        const int p = *s.dev_valid.begin();
        hexir_status_t st =
            hexir_buffer_read(s.dev[p], h, static_cast<size_t>(s.bytes));
        if (st != HEXIR_OK)
          return st;
      } else {
        std::memset(h, 0, static_cast<size_t>((s.bytes + 7) / 8 * 8));
      }
      s.host_valid = true;
    }
    *out = reinterpret_cast<const uint8_t *>(s.host);
    return HEXIR_OK;
  }

  // Storage for slot s's host copy, contents undefined: a page-locked block
  // when the execute has a GPU to copy to or from, else ordinary memory.
  double *host_storage(Slot &s) {
    const size_t bytes = static_cast<size_t>((s.bytes + 7) / 8 * 8);
    if (s.host)
      return s.host;
    void *p = cuda.empty() ? nullptr : pinned_take(bytes, cuda.front()->state->context);
    if (p) {
      pinned.emplace_back(p, bytes);
      s.host = static_cast<double *>(p);
    } else {
      s.host_own.reset(new double[bytes / 8]);
      s.host = s.host_own.get();
    }
    return s.host;
  }

  // The destination of a dispatch becomes valid only where it is written.
  void written_on_device(Slot &s, int o) {
    drop_borrowed(s);
    s.zero = false;
    s.rodata = nullptr;
    s.host_valid = false;
    s.dev_valid.clear();
    s.dev_valid.insert(o);
  }
  // nullptr when the storage cannot be had (an injected fault; a real
  // shortage throws std::bad_alloc, caught at the C ABI).
  double *written_on_host(Slot &s) {
    if (fault_hit(FaultSite::Alloc))
      return nullptr;
    drop_borrowed(s);
    double *h = host_storage(s);
    s.zero = false;
    s.rodata = nullptr;
    s.host_valid = true;
    s.dev_valid.clear();
    return h;
  }

  // ---- dispatch ----------------------------------------------------------

  KernelLib *library(uint32_t index, int o) {
    auto key = std::make_pair(index, o);
    auto it = libs.find(key);
    if (it != libs.end())
      return it->second;
    const hexir_executable_entry_t &exe = exes[index];
    std::string error;
    KernelLib *lib = library_for_image(cuda[o]->state,
                                       exe_base + exe.image_offset,
                                       exe.image_size, &error);
    if (!lib)
      report(std::string("kernel '") + exe.name + "': " + error);
    libs[key] = lib;
    return lib;
  }

  Span *begin_span(CudaDevice *dev) {
    const Driver &d = driver();
    ContextGuard g(dev->state->context);
    Span sp;
    sp.device = dev;
    if (d.EventCreate(&sp.start, CU_EVENT_DEFAULT) != CUDA_SUCCESS ||
        d.EventCreate(&sp.stop, CU_EVENT_DEFAULT) != CUDA_SUCCESS)
      return nullptr;
    d.EventRecord(sp.start, dev->stream);
    spans.push_back(sp);
    return &spans.back();
  }
  void end_span(Span *sp) {
    if (!sp)
      return;
    ContextGuard g(sp->device->state->context);
    driver().EventRecord(sp->stop, sp->device->stream);
  }

  static uint64_t elems(const hexir_executable_entry_t &e) {
    return static_cast<uint64_t>(e.m) * e.n;
  }

  // Buffer sizes against the kernel's extents.
  // Operands before the destination, by kernel kind.
  static bool is_activation(uint32_t kind) {
    return kind >= HEXIR_KERNEL_LEAKY_RELU && kind <= HEXIR_KERNEL_MISH;
  }
  static int inputs_of(uint32_t kind) {
    if (is_activation(kind))
      return 1;
    switch (kind) {
    case HEXIR_KERNEL_RELU: return 1;
    case HEXIR_KERNEL_MATMUL_ADD:
    case HEXIR_KERNEL_MATMUL_ADD_RELU: return 3;
    default: return 2;
    }
  }
  static bool is_matmul(uint32_t kind) {
    return kind == HEXIR_KERNEL_MATMUL || kind == HEXIR_KERNEL_MATMUL_RELU ||
           kind == HEXIR_KERNEL_MATMUL_ADD || kind == HEXIR_KERNEL_MATMUL_ADD_RELU;
  }
  static uint32_t matmul_flags(uint32_t kind) {
    return kind == HEXIR_KERNEL_MATMUL_RELU || kind == HEXIR_KERNEL_MATMUL_ADD_RELU
               ? HEXIR_MATMUL_RELU
               : 0u;
  }
  static bool has_addend(uint32_t kind) {
    return kind == HEXIR_KERNEL_MATMUL_ADD || kind == HEXIR_KERNEL_MATMUL_ADD_RELU;
  }

  hexir_status_t check_sizes(const hexir_executable_entry_t &exe,
                             Slot *const *args, uint64_t argc) {
    if (exe.elem_size != sizeof(double))
      return HEXIR_ERROR_UNIMPLEMENTED;
    const uint64_t mn = elems(exe) * 8;
    switch (exe.kind) {
    case HEXIR_KERNEL_MATMUL:
    case HEXIR_KERNEL_MATMUL_RELU:
      if (argc != 3)
        return HEXIR_ERROR_INVALID_MODULE;
      if (args[0]->bytes < static_cast<uint64_t>(exe.m) * exe.k * 8 ||
          args[1]->bytes < static_cast<uint64_t>(exe.k) * exe.n * 8 ||
          args[2]->bytes < mn)
        return HEXIR_ERROR_INVALID_MODULE;
      return HEXIR_OK;
    case HEXIR_KERNEL_MATMUL_ADD:
    case HEXIR_KERNEL_MATMUL_ADD_RELU:
      if (argc != 4)
        return HEXIR_ERROR_INVALID_MODULE;
      if (args[0]->bytes < static_cast<uint64_t>(exe.m) * exe.k * 8 ||
          args[1]->bytes < static_cast<uint64_t>(exe.k) * exe.n * 8 ||
          args[2]->bytes < mn || args[3]->bytes < mn)
        return HEXIR_ERROR_INVALID_MODULE;
      return HEXIR_OK;
    case HEXIR_KERNEL_ADD:
      if (argc != 3)
        return HEXIR_ERROR_INVALID_MODULE;
      if (args[0]->bytes < mn || args[1]->bytes < mn || args[2]->bytes < mn)
        return HEXIR_ERROR_INVALID_MODULE;
      return HEXIR_OK;
    case HEXIR_KERNEL_RELU:
    case HEXIR_KERNEL_LEAKY_RELU:
    case HEXIR_KERNEL_ELU:
    case HEXIR_KERNEL_SIGMOID:
    case HEXIR_KERNEL_TANH:
    case HEXIR_KERNEL_SOFTMAX:
    case HEXIR_KERNEL_GELU:
    case HEXIR_KERNEL_SWISH:
    case HEXIR_KERNEL_MISH:
      if (argc != 2)
        return HEXIR_ERROR_INVALID_MODULE;
      if (args[0]->bytes < mn || args[1]->bytes < mn)
        return HEXIR_ERROR_INVALID_MODULE;
      return HEXIR_OK;
    default:
      return HEXIR_ERROR_UNIMPLEMENTED;
    }
  }

  hexir_status_t run_host(const hexir_executable_entry_t &exe, Slot *const *args) {
    const int inputs = inputs_of(exe.kind);
    const uint8_t *in[3] = {nullptr, nullptr, nullptr};
    hexir_status_t st = HEXIR_OK;
    for (int i = 0; i < inputs && st == HEXIR_OK; ++i)
      st = on_host(*args[i], &in[i]);
    if (st != HEXIR_OK)
      return st;
    Slot &dst = *args[inputs];
    // Inputs may alias the destination slot only in a malformed module; copy
    // them out first so writing cannot corrupt them.
    std::vector<double> keep[3];
    for (int i = 0; i < inputs; ++i)
      if (args[i] == &dst) {
        keep[i].assign(reinterpret_cast<const double *>(in[i]),
                       reinterpret_cast<const double *>(in[i]) + args[i]->bytes / 8);
        in[i] = reinterpret_cast<const uint8_t *>(keep[i].data());
      }
    const double *a = reinterpret_cast<const double *>(in[0]);
    const double *b = reinterpret_cast<const double *>(in[1]);
    const double *d = reinterpret_cast<const double *>(in[2]);
    double *c = written_on_host(dst);
    if (!c)
      return HEXIR_ERROR_OUT_OF_MEMORY;
    switch (exe.kind) {
    case HEXIR_KERNEL_MATMUL:
      cpu_matmul_f64(a, b, c, exe.m, exe.n, exe.k);
      break;
    case HEXIR_KERNEL_MATMUL_RELU:
      cpu_matmul_f64(a, b, c, exe.m, exe.n, exe.k);
      cpu_relu_f64(c, c, elems(exe));
      break;
    case HEXIR_KERNEL_MATMUL_ADD:
    case HEXIR_KERNEL_MATMUL_ADD_RELU:
      cpu_matmul_f64(a, b, c, exe.m, exe.n, exe.k);
      cpu_add_f64(c, d, c, elems(exe));
      if (exe.kind == HEXIR_KERNEL_MATMUL_ADD_RELU)
        cpu_relu_f64(c, c, elems(exe));
      break;
    case HEXIR_KERNEL_ADD:
      cpu_add_f64(a, b, c, elems(exe));
      break;
    case HEXIR_KERNEL_RELU:
      cpu_relu_f64(a, c, elems(exe));
      break;
    default:
      cpu_activation_f64(exe.kind, a, c, exe.m, exe.n);
      break;
    }
    return HEXIR_OK;
  }

  // A large matmul whose operands still live on the host, or whose result is
  // the one being captured, runs as a pipeline on two streams: uploads on the
  // device's copy stream, kernels on its main stream, downloads of finished
  // rows on the copy stream.
  //   - Weight still on the host (and the one-shot launch has no k split):
  //     phase 1 runs k in [0, K1) over all rows in pieces of growing length,
  //     each piece's rows of w (and columns of a) uploading while the
  //     previous piece computes, every launch continuing the previous one's
  //     sums; phase 2 runs k in [K1, K) per row chunk, continuing from phase
  //     1, with the relu, and each finished chunk downloads while the next
  //     computes.  Only the first, short piece's upload and the last chunk's
  //     download are exposed.
  //   - Otherwise: w whole first, then row chunks of a upload while the
  //     previous chunk computes, and finished chunks download.
  // Both perform each element's operations in the one-shot order (no k
  // split, or the one-shot's own split for every row chunk), so results are
  // bit-identical to a single launch.
  static constexpr uint64_t kPipelineBytes = 64ull << 20;
  // Row chunks: 1/4, 1/4, 1/4, 1/8, 1/8 of the rows (128-row multiples), so
  // the one download left exposed after the last kernel is an eighth.
  static constexpr uint32_t kPipelineChunks = 5;
  static void pipeline_chunk(uint64_t m, uint32_t i, uint64_t *begin,
                             uint64_t *rows) {
    static const uint32_t eighths[kPipelineChunks + 1] = {0, 2, 4, 6, 7, 8};
    auto bound = [&](uint32_t j) {
      return j == kPipelineChunks ? m : (m * eighths[j] / 8) / 128 * 128;
    };
    *begin = bound(i);
    *rows = bound(i + 1) - *begin;
  }
  static constexpr uint32_t kPieceMinK = 2048;

  // Slot s's bytes are on the host and would be uploaded by this dispatch.
  bool host_upload(const Slot &s, int o) {
    ModuleState *ms = s.rodata ? module_state(module) : nullptr;
    const bool kept = ms && ms->keep_constants.load();  // uploaded once, whole
    return !s.dev_valid.count(o) && !s.zero && (s.rodata || s.host_valid) &&
           s.bytes >= kPipelineBytes && !kept;
  }

  bool want_pipeline(const hexir_executable_entry_t &exe, Slot *const *args,
                     int o, bool *upload_a, bool *upload_w, bool *stream_out) {
    if (exe.kind != HEXIR_KERNEL_MATMUL && exe.kind != HEXIR_KERNEL_MATMUL_RELU)
      return false;
    Slot &dst = *args[2];
    if (&dst == args[0] || &dst == args[1] || args[0] == args[1] ||
        exe.m < 1024)
      return false;
    *upload_a = host_upload(*args[0], o);
    *upload_w = host_upload(*args[1], o) && exe.k >= kPieceMinK;
    *stream_out = capture_out && capture_size && current_pc == last_dispatch_pc &&
                  dst.bytes >= kPipelineBytes;
    return *upload_a || *upload_w || *stream_out;
  }

  // A matmul shape that want_pipeline could split into row chunks, whatever
  // its operands' residency.  Every launch of such a dispatch, pipelined or
  // not (constants kept on the GPU, operands already there), plans without
  // stream-K, whose sums follow the whole tile set: so its bits do not
  // depend on where its operands were.
  static bool row_chunk_shape(const hexir_executable_entry_t &exe) {
    if (exe.kind != HEXIR_KERNEL_MATMUL && exe.kind != HEXIR_KERNEL_MATMUL_RELU)
      return false;
    const uint64_t a = uint64_t{exe.m} * exe.k * 8, w = uint64_t{exe.k} * exe.n * 8,
                   c = uint64_t{exe.m} * exe.n * 8;
    return exe.m >= 1024 && (a >= kPipelineBytes || c >= kPipelineBytes ||
                             (w >= kPipelineBytes && exe.k >= kPieceMinK));
  }

  // Bounds of phase 1's k pieces over [0, k1): weight_stream_bounds.
  static std::vector<uint32_t> k_piece_bounds(uint32_t k1) {
    return weight_stream_bounds(k1);
  }

  hexir_status_t run_pipelined(uint32_t index, int o, Slot *const *args,
                               bool upload_a, bool upload_w, bool stream_out) {
    const hexir_executable_entry_t &exe = exes[index];
    KernelLib *lib = library(index, o);
    if (!lib)
      return HEXIR_ERROR_DEVICE;
    CudaDevice *dev = cuda[o];
    const Driver &d = driver();
    Slot &as = *args[0];
    Slot &ws = *args[1];
    Slot &dst = *args[2];
    CUdeviceptr a_dev = 0, w_dev = 0, c_dev = 0;
    hexir_status_t st = upload_w ? writable_on(ws, o, ws.bytes, &w_dev)
                                 : on_device(ws, o, &w_dev);
    if (st == HEXIR_OK)
      st = upload_a ? writable_on(as, o, as.bytes, &a_dev) : on_device(as, o, &a_dev);
    if (st == HEXIR_OK)
      st = writable_on(dst, o, dst.bytes, &c_dev);
    if (st != HEXIR_OK)
      return st;
    const uint32_t relu =
        exe.kind == HEXIR_KERNEL_MATMUL_RELU ? HEXIR_MATMUL_RELU : 0u;
    // Row chunks and k pieces reproduce the one-shot launch's sums only
    // for a data-parallel or split-K plan (row_chunk_shape).
    const MatmulPlan whole = plan_matmul(
        dev->state, reinterpret_cast<const double *>(a_dev),
        reinterpret_cast<const double *>(w_dev),
        reinterpret_cast<const double *>(c_dev), exe.m, exe.n, exe.k,
        relu | HEXIR_MATMUL_NO_STREAM_K);
    const bool pieces = upload_w && whole.split_k == 1;
    if (upload_w && !pieces) {
      // The one-shot launch splits k: upload w whole before the row chunks.
      if ((st = copy_range_to(ws, 0, ws.bytes, o, w_dev)) != HEXIR_OK)
        return st;
      ws.dev_valid.insert(o);
    }
    CUstream cs = dev->copy_stream();
    if (!cs)
      return HEXIR_ERROR_DEVICE;
    ContextGuard guard(dev->state->context);
    std::vector<CUevent> events;
    auto event = [&](CUstream on) -> CUevent {
      CUevent ev = nullptr;
      if (d.EventCreate(&ev, CU_EVENT_DISABLE_TIMING) != CUDA_SUCCESS)
        return nullptr;
      d.EventRecord(ev, on);
      events.push_back(ev);
      return ev;
    };
    auto release_events = [&] {
      for (CUevent ev : events)
        d.EventDestroy(ev);  // released once complete
    };
    // The copy stream starts after everything queued on the main stream
    // (the buffers may be reused pool blocks).
    CUevent ready = event(dev->stream);
    if (!ready)
      return HEXIR_ERROR_DEVICE;
    d.StreamWaitEvent(cs, ready, 0);
    Span *span = begin_span(dev);
    const uint64_t K = exe.k, N = exe.n;
    const uint64_t row_a = K * 8;
    const uint64_t row_c = N * 8;
    uint64_t r0[kPipelineChunks], rows[kPipelineChunks];
    for (uint32_t i = 0; i < kPipelineChunks; ++i)
      pipeline_chunk(exe.m, i, &r0[i], &rows[i]);
    auto host_bytes = [&](Slot &s, uint64_t off, uint64_t bytes) {
      return s.rodata ? rodata_source(s, off, bytes)
                      : reinterpret_cast<const uint8_t *>(s.host) + off;
    };
    // Uploads of w's rows [k0, k1) and of a's columns [k0, k1) for rows
    // [ra, ra + nr), on the copy stream.
    auto upload_w_rows = [&](uint64_t k0, uint64_t k1) -> bool {
      const uint64_t off = k0 * row_c, bytes = (k1 - k0) * row_c;
      return d.MemcpyHtoDAsync(w_dev + off, host_bytes(ws, off, bytes), bytes,
                               cs) == CUDA_SUCCESS;
    };
    auto upload_a_cols = [&](uint64_t ra, uint64_t nr, uint64_t k0,
                             uint64_t k1) -> bool {
      if (!nr)
        return true;
      CUDA_MEMCPY2D cp;
      std::memset(&cp, 0, sizeof(cp));
      cp.srcMemoryType = CU_MEMORYTYPE_HOST;
      cp.srcHost = host_bytes(as, ra * row_a, nr * row_a) + k0 * 8;
      cp.srcPitch = row_a;
      cp.dstMemoryType = CU_MEMORYTYPE_DEVICE;
      cp.dstDevice = a_dev + ra * row_a + k0 * 8;
      cp.dstPitch = row_a;
      cp.WidthInBytes = (k1 - k0) * 8;
      cp.Height = nr;
      return d.Memcpy2DAsync(&cp, cs) == CUDA_SUCCESS;
    };
    auto fail_copy = [&]() {
      report("host to device copy failed (pipelined dispatch)");
      release_events();
      return HEXIR_ERROR_DEVICE;
    };
    auto launch = [&](uint64_t ra, uint64_t nr, uint64_t k0, uint64_t k1,
                      uint32_t flags, bool cont,
                      CUstream on = nullptr) -> hexir_status_t {
      std::string error;
      double *c = reinterpret_cast<double *>(c_dev + ra * row_c);
      hexir_status_t ls = launch_matmul(
          dev->state, lib, reinterpret_cast<const double *>(a_dev + ra * row_a + k0 * 8),
          reinterpret_cast<const double *>(w_dev + k0 * row_c), c,
          static_cast<uint32_t>(nr), exe.n, static_cast<uint32_t>(k1 - k0),
          flags | HEXIR_MATMUL_SPLIT_K(1), on ? on : dev->stream, &error, exe.k,
          cont ? c : nullptr);
      if (ls != HEXIR_OK)
        report(std::string("kernel '") + exe.name + "': " + error);
      return ls;
    };
    std::vector<CUevent> c_ready(kPipelineChunks, nullptr);
    // The row chunks are independent: odd ones run on the side stream (after
    // everything queued on the main stream so far), so each chunk's last
    // wave of tiles overlaps the next one's first.  The main stream joins it
    // after the chunks.
    CUstream side = dev->side_stream();
    bool side_started = false;
    // Called before the first chunk is queued: the side stream starts after
    // everything on the main stream up to here.
    auto fork_side = [&]() {
      if (!side)
        return;
      CUevent fork = event(dev->stream);
      if (fork && d.StreamWaitEvent(side, fork, 0) == CUDA_SUCCESS)
        side_started = true;
    };
    auto chunk_stream = [&](uint32_t i) -> CUstream {
      return side_started && i % 2 == 1 ? side : dev->stream;
    };
    auto join_side = [&]() {
      if (side_started) {
        CUevent done = event(side);
        if (done)
          d.StreamWaitEvent(dev->stream, done, 0);
      }
    };
    if (pieces) {
      const uint64_t k1 = K / 2 / 32 * 32;
      const std::vector<uint32_t> b = k_piece_bounds(static_cast<uint32_t>(k1));
      std::vector<CUevent> piece_ready;
      for (size_t j = 0; j + 1 < b.size(); ++j) {
        if (!upload_w_rows(b[j], b[j + 1]) ||
            (upload_a && !upload_a_cols(0, exe.m, b[j], b[j + 1])))
          return fail_copy();
        piece_ready.push_back(event(cs));
      }
      if (!upload_w_rows(k1, K))
        return fail_copy();
      std::vector<CUevent> chunk_ready(kPipelineChunks, nullptr);
      CUevent w_ready = event(cs);
      for (uint32_t i = 0; i < kPipelineChunks; ++i) {
        if (upload_a && !upload_a_cols(r0[i], rows[i], k1, K))
          return fail_copy();
        chunk_ready[i] = upload_a ? event(cs) : w_ready;
      }
      for (size_t j = 0; j + 1 < b.size(); ++j) {
        d.StreamWaitEvent(dev->stream, piece_ready[j], 0);
        if ((st = launch(0, exe.m, b[j], b[j + 1], 0u, j > 0)) != HEXIR_OK) {
          release_events();
          return st;
        }
      }
      fork_side();
      for (uint32_t i = 0; i < kPipelineChunks; ++i) {
        if (!rows[i])
          continue;
        CUstream on = chunk_stream(i);
        d.StreamWaitEvent(on, chunk_ready[i], 0);
        if ((st = launch(r0[i], rows[i], k1, K, relu, k1 > 0, on)) != HEXIR_OK) {
          join_side();
          release_events();
          return st;
        }
        if (stream_out)
          c_ready[i] = event(on);
      }
      join_side();
    } else {
      std::vector<CUevent> a_ready(kPipelineChunks, nullptr);
      for (uint32_t i = 0; i < kPipelineChunks; ++i) {
        if (!upload_a || !rows[i])
          continue;
        const uint64_t off = r0[i] * row_a, bytes = rows[i] * row_a;
        if (d.MemcpyHtoDAsync(a_dev + off, host_bytes(as, off, bytes), bytes,
                              cs) != CUDA_SUCCESS)
          return fail_copy();
        a_ready[i] = event(cs);
      }
      // Every chunk uses the k split the whole matmul would use, so each
      // element is summed exactly as by the one-shot launch.
      const uint32_t flags = relu | HEXIR_MATMUL_SPLIT_K(whole.split_k);
      fork_side();
      for (uint32_t i = 0; i < kPipelineChunks; ++i) {
        if (!rows[i])
          continue;
        CUstream on = chunk_stream(i);
        if (a_ready[i])
          d.StreamWaitEvent(on, a_ready[i], 0);
        std::string error;
        st = launch_matmul(
            dev->state, lib,
            reinterpret_cast<const double *>(a_dev + r0[i] * row_a),
            reinterpret_cast<const double *>(w_dev),
            reinterpret_cast<double *>(c_dev + r0[i] * row_c),
            static_cast<uint32_t>(rows[i]), exe.n, exe.k, flags, on, &error);
        if (st != HEXIR_OK) {
          report(std::string("kernel '") + exe.name + "': " + error);
          join_side();
          release_events();
          return st;
        }
        if (stream_out)
          c_ready[i] = event(on);
      }
      join_side();
    }
    end_span(span);
    if (stream_out) {
      // Rows out to the capture buffer as their chunk finishes.
      for (uint32_t i = 0; i < kPipelineChunks; ++i) {
        if (!c_ready[i])
          continue;
        const uint64_t begin = r0[i] * row_c;
        if (begin >= capture_size)
          break;
        const uint64_t bytes = std::min<uint64_t>(rows[i] * row_c,
                                                  capture_size - begin);
        d.StreamWaitEvent(cs, c_ready[i], 0);
        if (d.MemcpyDtoHAsync(static_cast<uint8_t *>(capture_out) + begin,
                              c_dev + begin, bytes, cs) != CUDA_SUCCESS) {
          release_events();
          return HEXIR_ERROR_DEVICE;
        }
        if (capture_user) {
          // Outlives this dispatch: the chunk's host copy waits on it.
          CUevent landed = nullptr;
          if (d.EventCreate(&landed, CU_EVENT_DISABLE_TIMING) != CUDA_SUCCESS ||
              d.EventRecord(landed, cs) != CUDA_SUCCESS) {
            if (landed)
              d.EventDestroy(landed);
            release_events();
            return HEXIR_ERROR_DEVICE;
          }
          staged_chunks.emplace_back(begin, bytes, landed);
        }
      }
      capture_done = true;
    }
    // The main stream covers the copies from here on.
    CUevent copies_done = event(cs);
    if (copies_done)
      d.StreamWaitEvent(dev->stream, copies_done, 0);
    release_events();
    if (upload_a)
      as.dev_valid.insert(o);
    if (upload_w)
      ws.dev_valid.insert(o);
    written_on_device(dst, o);
    return HEXIR_OK;
  }

  // ---- constants uploaded ahead ---------------------------------------------

  // A later dispatch's constant starts uploading only once it is at least
  // this large (smaller ones cost less than the bookkeeping), and at most
  // kPrefetchCapBytes are in flight or waiting to be adopted.
  static constexpr uint64_t kPrefetchMinBytes = 4ull << 20;
  static constexpr uint64_t kPrefetchCapBytes = 8ull << 30;

  // The single GPU (program ordinal) an executable runs on through the
  // kernel library, or -1 (host, reference-convention image, row-sharded).
  int single_gpu(uint64_t index) const {
    if (index >= exe_count || exes[index].device != HEXIR_DEVICE_CUDA ||
        !launches || index >= launch_count)
      return -1;
    const hexir_launch_entry_t &L = launches[index];
    if (L.abi != HEXIR_LAUNCH_ABI_V1 || !(L.flags & HEXIR_LAUNCH_FLAG_LIBRARY) ||
        L.device_count > 1 || L.device_first >= cuda.size())
      return -1;
    return static_cast<int>(L.device_first);
  }

  // After a dispatch is queued: the constants that later single-GPU
  // dispatches of this entry read start uploading on their GPU's copy
  // stream, behind the uploads the queued dispatch makes there, so they
  // cross PCIe while its kernel runs instead of in front of the kernel
  // that needs them.  A program binds a constant (CONST) just before its
  // first use, so the scan records CONSTs as it meets them and matches
  // DISPATCH operands against them; it stops at END.
  hexir_status_t prefetch_ahead(uint64_t pc) {
    if (cuda.empty() || !program)
      return HEXIR_OK;
    ModuleState *ms = module_state(module);
    if (ms && ms->keep_constants.load())
      return HEXIR_OK;  // kept constants are uploaded once, whole
    std::map<uint64_t, std::pair<uint64_t, uint64_t>> const_of;  // slot -> (offset, bytes)
    while (pc + sizeof(hexir_command_header_t) <= program_size) {
      hexir_command_header_t h;
      std::memcpy(&h, program + pc, sizeof(h));
      const uint64_t at = pc + sizeof(h);
      const uint64_t next = at + static_cast<uint64_t>(h.operand_count) * 8;
      if (next > program_size || h.kind == HEXIR_CMD_END)
        break;
      auto operand = [&](uint32_t i) {
        uint64_t v;
        std::memcpy(&v, program + at + 8ull * i, 8);
        return v;
      };
      if (h.kind == HEXIR_CMD_CONST && h.operand_count == 3) {
        const uint64_t offset = operand(1), bytes = operand(2);
        if (offset <= rodata_size && bytes <= rodata_size - offset)
          const_of[operand(0)] = {offset, bytes};
      } else if (h.kind == HEXIR_CMD_ALLOC && h.operand_count >= 1) {
        const_of.erase(operand(0));
      } else if (h.kind == HEXIR_CMD_DISPATCH && h.operand_count >= 3) {
        const int o = single_gpu(operand(0));
        // Inputs only: the last operand is the destination.
        for (uint32_t i = 2; o >= 0 && i + 1 < h.operand_count; ++i) {
          auto it = const_of.find(operand(i));
          if (it == const_of.end())
            continue;
          const uint64_t offset = it->second.first, bytes = it->second.second;
          if (bytes < kPrefetchMinBytes ||
              prefetched.count({offset, o}) ||
              prefetched_bytes + bytes > kPrefetchCapBytes)
            continue;
          hexir_status_t st = start_prefetch(offset, bytes, o);
          if (st != HEXIR_OK)
            return st;
        }
      }
      pc = next;
    }
    return HEXIR_OK;
  }

  hexir_status_t start_prefetch(uint64_t offset, uint64_t bytes, int o) {
    CudaDevice *dev = cuda[o];
    CUstream cs = dev->copy_stream();
    if (!cs)
      return HEXIR_OK;  // no copy stream: the dispatch uploads as usual
    hexir_buffer_t *b = nullptr;
    if (dev->allocate_pooled(bytes, &b) != HEXIR_OK)
      return HEXIR_OK;  // no room ahead of time: the dispatch uploads it
    const Driver &d = driver();
    ContextGuard guard(dev->state->context);
    Slot view;
    view.rodata = rodata + offset;
    CUevent ready = nullptr;
    CUresult r = d.MemcpyHtoDAsync(reinterpret_cast<CUdeviceptr>(b->impl),
                                   rodata_source(view, 0, bytes), bytes, cs);
    if (r == CUDA_SUCCESS)
      r = d.EventCreate(&ready, CU_EVENT_DISABLE_TIMING);
    if (r == CUDA_SUCCESS)
      r = d.EventRecord(ready, cs);
    if (r != CUDA_SUCCESS) {
      d.StreamSynchronize(cs);
      if (ready)
        d.EventDestroy(ready);
      hexir_buffer_release(b);
      report(cuda_message("constant upload ahead of its dispatch", r));
      return HEXIR_ERROR_DEVICE;
    }
    prefetched[{offset, o}] = Prefetched{bytes, b, ready};
    prefetched_bytes += bytes;
    if (trace)
      std::fprintf(stderr, "hexir: constant at %llu (%llu bytes) uploading "
                   "ahead to cuda:%d\n", static_cast<unsigned long long>(offset),
                   static_cast<unsigned long long>(bytes), o);
    return HEXIR_OK;
  }

  // A CONST just bound slot s to RODATA at `offset`: where that constant was
  // uploaded ahead, the slot takes the buffer, and the GPU's stream waits
  // for the upload before anything that reads it.
  hexir_status_t adopt_prefetched(Slot &s, uint64_t offset) {
    for (auto it = prefetched.begin(); it != prefetched.end();) {
      if (it->first.first != offset || it->second.bytes != s.bytes) {
        ++it;
        continue;
      }
      const int o = it->first.second;
      CudaDevice *dev = cuda[o];
      ContextGuard guard(dev->state->context);
      const CUresult r = driver().StreamWaitEvent(dev->stream, it->second.ready, 0);
      driver().EventDestroy(it->second.ready);
      if (r != CUDA_SUCCESS) {
        hexir_buffer_release(it->second.buffer);
        prefetched_bytes -= it->second.bytes;
        prefetched.erase(it);
        report(cuda_message("waiting for a constant uploaded ahead", r));
        return HEXIR_ERROR_DEVICE;
      }
      s.dev[o] = it->second.buffer;
      s.dev_valid.insert(o);
      prefetched_bytes -= it->second.bytes;
      it = prefetched.erase(it);
    }
    return HEXIR_OK;
  }

  hexir_status_t run_device(uint32_t index, int o, Slot *const *args) {
    const hexir_executable_entry_t &exe = exes[index];
    bool upload_a = false, upload_w = false, stream_out = false;
    if (want_pipeline(exe, args, o, &upload_a, &upload_w, &stream_out))
      return run_pipelined(index, o, args, upload_a, upload_w, stream_out);
    KernelLib *lib = library(index, o);
    if (!lib)
      return HEXIR_ERROR_DEVICE;
    CudaDevice *dev = cuda[o];
    const int inputs = inputs_of(exe.kind);
    CUdeviceptr in[3] = {0, 0, 0}, out = 0;
    Slot &dst = *args[inputs];
    hexir_status_t st = HEXIR_OK;
    bool aliased = false;
    for (int i = 0; i < inputs && st == HEXIR_OK; ++i) {
      st = on_device(*args[i], o, &in[i]);
      aliased |= args[i] == &dst;
    }
    if (st != HEXIR_OK)
      return st;
    if (aliased) {
      // Malformed aliasing: give the destination a fresh buffer.
      CUdeviceptr tmp = 0;
      if ((st = temp_on(o, dst.bytes, &tmp)) != HEXIR_OK)
        return st;
      out = tmp;
    } else if ((st = writable_on(dst, o, dst.bytes, &out)) != HEXIR_OK) {
      return st;
    }
    std::string error;
    ContextGuard guard(dev->state->context);
    Span *span = begin_span(dev);
    const double *a = reinterpret_cast<const double *>(in[0]);
    const double *b = reinterpret_cast<const double *>(in[1]);
    double *c = reinterpret_cast<double *>(out);
    switch (exe.kind) {
    case HEXIR_KERNEL_MATMUL:
    case HEXIR_KERNEL_MATMUL_RELU:
    case HEXIR_KERNEL_MATMUL_ADD:
    case HEXIR_KERNEL_MATMUL_ADD_RELU:
      st = launch_matmul(dev->state, lib, a, b, c, exe.m, exe.n, exe.k,
                         matmul_flags(exe.kind) |
                             (row_chunk_shape(exe) ? HEXIR_MATMUL_NO_STREAM_K : 0u),
                         dev->stream, &error, 0, nullptr,
                         has_addend(exe.kind)
                             ? reinterpret_cast<const double *>(in[2])
                             : nullptr);
      break;
    case HEXIR_KERNEL_ADD:
      st = launch_add(dev->state, lib, a, b, c, elems(exe), dev->stream, &error);
      break;
    case HEXIR_KERNEL_RELU:
      st = launch_relu(dev->state, lib, a, c, elems(exe), dev->stream, &error);
      break;
    default:
      st = launch_activation(dev->state, lib, exe.kind, a, c, exe.m, exe.n,
                             dev->stream, &error);
      break;
    }
    end_span(span);
    if (st != HEXIR_OK) {
      report(std::string("kernel '") + exe.name + "': " + error);
      return st;
    }
    if (out != reinterpret_cast<CUdeviceptr>(dst.dev.count(o) ? dst.dev[o]->impl
                                                              : nullptr)) {
      CUdeviceptr home = 0;
      if ((st = writable_on(dst, o, dst.bytes, &home)) != HEXIR_OK)
        return st;
      driver().MemcpyDtoDAsync(home, out, dst.bytes, dev->stream);
    }
    written_on_device(dst, o);
    return HEXIR_OK;
  }

  hexir_status_t run_sharded(uint32_t index, int first, int count,
                             Slot *const *args) {
    const hexir_executable_entry_t &exe = exes[index];
    const Nccl &nc = nccl();
    std::vector<int> ordinals;
    for (int r = 0; r < count; ++r)
      ordinals.push_back(cuda[first + r]->ordinal);
    std::vector<ncclComm_t> comms;
    std::string error;
    hexir_status_t st = comms_for(ordinals, &comms, &error);
    if (st != HEXIR_OK) {
      report(std::string("kernel '") + exe.name + "': " + error);
      return st;
    }
    const bool matmul = is_matmul(exe.kind);
    const int inputs = inputs_of(exe.kind);
    Slot &dst = *args[inputs];
    for (int i = 0; i < inputs; ++i)
      if (&dst == args[i])
        return HEXIR_ERROR_INVALID_MODULE;
    for (int r = 0; r < count; ++r)
      if (!library(index, first + r))
        return HEXIR_ERROR_DEVICE;
    CudaDevice *root = cuda[first];
    Span *span = begin_span(root);
    // Every stream of the range starts after the work queued on the root.
    for (int r = 1; r < count; ++r)
      if ((st = order_after(root, cuda[first + r])) != HEXIR_OK)
        return st;

    // Weight of a matmul: valid on the root, then broadcast over NVLink.
    std::vector<CUdeviceptr> w(count, 0);
    if (matmul) {
      Slot &ws = *args[1];
      if ((st = on_device(ws, first, &w[0])) != HEXIR_OK)
        return st;
      bool everywhere = true;
      for (int r = 1; r < count; ++r)
        everywhere &= ws.dev_valid.count(first + r) > 0;
      // The broadcast writes every peer's copy, so those must be writable.
      for (int r = 1; r < count; ++r)
        if ((st = everywhere ? buffer_on(ws, first + r, ws.bytes, &w[r])
                             : writable_on(ws, first + r, ws.bytes, &w[r])) !=
            HEXIR_OK)
          return st;
      if (!everywhere) {
        const size_t elemsw = static_cast<size_t>(exe.k) * exe.n;
        if (fault_hit(FaultSite::Nccl)) {
          report("ncclBroadcast (weight): injected fault (HEXIR_FAULT)");
          return HEXIR_ERROR_DEVICE;
        }
        nc.GroupStart();
        for (int r = 0; r < count; ++r)
          nc.Broadcast(reinterpret_cast<void *>(w[r]), reinterpret_cast<void *>(w[r]),
                       elemsw, ncclDouble, 0, comms[r],
                       reinterpret_cast<cudaStream_t>(cuda[first + r]->stream));
        ncclResult_t nr = nc.GroupEnd();
        if (nr != ncclSuccess) {
          report(nccl_message("ncclBroadcast (weight)", nr));
          return HEXIR_ERROR_DEVICE;
        }
        for (int r = 1; r < count; ++r)
          ws.dev_valid.insert(first + r);
      }
    }

    CUdeviceptr c_root = 0;
    if ((st = writable_on(dst, first, dst.bytes, &c_root)) != HEXIR_OK)
      return st;
    const uint64_t row_out = static_cast<uint64_t>(exe.n) * 8;
    // The row-split inputs and their row sizes: a (and the addend) of a
    // matmul, both operands of an add, the input of a relu.
    std::vector<std::pair<Slot *, uint64_t>> split_in;
    if (matmul) {
      split_in.emplace_back(args[0], static_cast<uint64_t>(exe.k) * 8);
      if (has_addend(exe.kind))
        split_in.emplace_back(args[2], row_out);
    } else {
      for (int i = 0; i < inputs; ++i)
        split_in.emplace_back(args[i], row_out);
    }
    std::vector<CUdeviceptr> c_part(count, 0);
    std::vector<uint64_t> begin(count), rows(count);
    std::vector<char> direct(count, 0);
    for (int r = 0; r < count; ++r) {
      hexir_shard_rows(exe.m, static_cast<uint32_t>(count),
                       static_cast<uint32_t>(r), &begin[r], &rows[r]);
      if (!rows[r])
        continue;
      const int o = first + r;
      CudaDevice *dev = cuda[o];
      // This shard's rows of the row-split inputs.
      CUdeviceptr x = 0, y = 0;
      for (size_t i = 0; i < split_in.size(); ++i) {
        Slot &in = *split_in[i].first;
        const uint64_t row_in = split_in[i].second;
        CUdeviceptr p = 0;
        if (in.dev_valid.count(o)) {
          p = reinterpret_cast<CUdeviceptr>(in.dev[o]->impl) + begin[r] * row_in;
        } else {
          if ((st = temp_on(o, rows[r] * row_in, &p)) != HEXIR_OK ||
              (st = copy_range_to(in, begin[r] * row_in, rows[r] * row_in, o,
                                  p)) != HEXIR_OK)
            return st;
        }
        (i == 0 ? x : y) = p;
      }
      // With peer access to the first GPU, the shard's kernel stores its rows
      // straight into the result there over NVLink, tile by tile as they are
      // computed; otherwise it writes a local block for the NCCL gather below.
      CUdeviceptr out = 0;
      direct[r] = r == 0 || peer_access(cuda[o], root);
      if (direct[r]) {
        out = c_root + begin[r] * row_out;
      } else if ((st = temp_on(o, rows[r] * row_out, &out)) != HEXIR_OK) {
        return st;
      }
      c_part[r] = out;
      ContextGuard guard(dev->state->context);
      KernelLib *lib = libs[std::make_pair(index, o)];
      const uint32_t m = static_cast<uint32_t>(rows[r]);
      const uint64_t count_elems = rows[r] * exe.n;
      switch (exe.kind) {
      case HEXIR_KERNEL_MATMUL:
      case HEXIR_KERNEL_MATMUL_RELU:
      case HEXIR_KERNEL_MATMUL_ADD:
      case HEXIR_KERNEL_MATMUL_ADD_RELU:
        // A shard is a row piece of one matmul: no stream-K, whose sums
        // would follow this shard's tile set rather than the rows'.
        st = launch_matmul(dev->state, lib, reinterpret_cast<const double *>(x),
                           reinterpret_cast<const double *>(w[r]),
                           reinterpret_cast<double *>(out), m, exe.n, exe.k,
                           matmul_flags(exe.kind) | HEXIR_MATMUL_NO_STREAM_K |
                               (r && direct[r] ? HEXIR_MATMUL_REMOTE_OUTPUT : 0u),
                           dev->stream, &error, 0, nullptr,
                           has_addend(exe.kind)
                               ? reinterpret_cast<const double *>(y)
                               : nullptr);
        break;
      case HEXIR_KERNEL_ADD:
        st = launch_add(dev->state, lib, reinterpret_cast<const double *>(x),
                        reinterpret_cast<const double *>(y),
                        reinterpret_cast<double *>(out), count_elems,
                        dev->stream, &error);
        break;
      case HEXIR_KERNEL_RELU:
        st = launch_relu(dev->state, lib, reinterpret_cast<const double *>(x),
                         reinterpret_cast<double *>(out), count_elems,
                         dev->stream, &error);
        break;
      default:
        st = launch_activation(dev->state, lib, exe.kind,
                               reinterpret_cast<const double *>(x),
                               reinterpret_cast<double *>(out), rows[r], exe.n,
                               dev->stream, &error);
        break;
      }
      if (st != HEXIR_OK) {
        report(std::string("kernel '") + exe.name + "' shard " +
               std::to_string(r) + ": " + error);
        // Shards already launched may still be storing into the root's
        // result: the root's stream (and the release of its buffers back to
        // the pool) must come after them.
        for (int j = 1; j < r; ++j)
          if (rows[j] && direct[j])
            order_after(cuda[first + j], root);
        return st;
      }
    }
    // The root's stream continues once every shard has finished; shards
    // that wrote directly only need that ordering, the rest send their rows.
    bool any_gather = false;
    for (int r = 1; r < count; ++r) {
      if (!rows[r])
        continue;
      if (direct[r]) {
        if ((st = order_after(cuda[first + r], root)) != HEXIR_OK)
          return st;
      } else {
        any_gather = true;
      }
    }
    if (any_gather) {
      if (fault_hit(FaultSite::Nccl)) {
        report("ncclSend/ncclRecv (rows): injected fault (HEXIR_FAULT)");
        return HEXIR_ERROR_DEVICE;
      }
      nc.GroupStart();
      for (int r = 1; r < count; ++r) {
        if (!rows[r] || direct[r])
          continue;
        nc.Send(reinterpret_cast<void *>(c_part[r]), rows[r] * exe.n, ncclDouble,
                0, comms[r],
                reinterpret_cast<cudaStream_t>(cuda[first + r]->stream));
        nc.Recv(reinterpret_cast<void *>(c_root + begin[r] * row_out),
                rows[r] * exe.n, ncclDouble, r, comms[0],
                reinterpret_cast<cudaStream_t>(root->stream));
      }
      ncclResult_t nr = nc.GroupEnd();
      if (nr != ncclSuccess) {
        report(nccl_message("row gather", nr));
        return HEXIR_ERROR_DEVICE;
      }
    }
    end_span(span);
    written_on_device(dst, first);
    return HEXIR_OK;
  }

  hexir_status_t dispatch(const uint64_t *ops, uint32_t count) {
    if (count < 2)
      return HEXIR_ERROR_INVALID_MODULE;
    const uint64_t index = ops[0], argc = ops[1];
    if (index >= exe_count || count != 2 + argc)
      return HEXIR_ERROR_INVALID_MODULE;
    const hexir_executable_entry_t &exe = exes[index];
    if (argc > 4)
      return HEXIR_ERROR_INVALID_MODULE;
    Slot *args[4] = {nullptr, nullptr, nullptr, nullptr};
    for (uint64_t i = 0; i < argc; ++i)
      if (!(args[i] = slot(ops[2 + i])))
        return HEXIR_ERROR_INVALID_MODULE;

    if (exe.device == HEXIR_DEVICE_CUDA) {
      if (cuda.empty()) {
        // The reference's refusal (interpreter.c:82-92), word for word.
        std::fprintf(stderr,
                     "hexir-run: kernel '%.32s' is placed on cuda but the "
                     "active device is %s\n",
                     exe.name, hexir_device_name(primary));
        return HEXIR_ERROR_DEVICE;
      }
      if (!exe.image_size) {
        std::fprintf(stderr,
                     "hexir-run: kernel '%.32s' is placed on cuda, but the "
                     "module carries a kernel descriptor rather than device "
                     "code, and there is nothing to launch\n",
                     exe.name);
        return HEXIR_ERROR_UNIMPLEMENTED;
      }
      if (static_cast<uint64_t>(exe.image_offset) + exe.image_size > exe_size)
        return HEXIR_ERROR_INVALID_MODULE;
      const hexir_launch_entry_t *L =
          (launches && index < launch_count) ? &launches[index] : nullptr;
      if (L && L->abi == HEXIR_LAUNCH_ABI_V1 &&
          (L->flags & HEXIR_LAUNCH_FLAG_LIBRARY)) {
        hexir_status_t st = check_sizes(exe, args, argc);
        if (st != HEXIR_OK)
          return st;
        const uint64_t first = L->device_first;
        const uint64_t n_dev = L->device_count ? L->device_count : 1;
        if (first + n_dev > cuda.size()) {
          std::fprintf(stderr,
                       "hexir-run: kernel '%.32s' is placed on cuda:%llu%s%s but "
                       "only %zu CUDA device(s) are open\n",
                       exe.name, static_cast<unsigned long long>(first),
                       n_dev > 1 ? "-" : "",
                       n_dev > 1 ? std::to_string(first + n_dev - 1).c_str() : "",
                       cuda.size());
          return HEXIR_ERROR_DEVICE;
        }
        if (trace)
          std::fprintf(stderr, "hexir: dispatch %.32s %s %ux%ux%u on cuda:%llu%s\n",
                       exe.name, hexir_kernel_kind_string(exe.kind), exe.m,
                       exe.n, exe.k, static_cast<unsigned long long>(first),
                       n_dev > 1 ? (" x" + std::to_string(n_dev)).c_str() : "");
        if (n_dev == 1)
          return run_device(static_cast<uint32_t>(index), static_cast<int>(first),
                            args);
        return run_sharded(static_cast<uint32_t>(index), static_cast<int>(first),
                           static_cast<int>(n_dev), args);
      }
      // An image following the reference convention: launch by entry name
      // with one device pointer per argument, on the first GPU.
      hexir_buffer_t *buffers[4];
      for (uint64_t i = 0; i < argc; ++i) {
        CUdeviceptr p = 0;
        hexir_status_t st;
        if (i + 1 == argc) {
          st = writable_on(*args[i], 0, args[i]->bytes, &p);
          if (st == HEXIR_OK && !args[i]->dev_valid.count(0))
            st = copy_range_to(*args[i], 0, args[i]->bytes, 0, p);
        } else {
          st = on_device(*args[i], 0, &p);
        }
        if (st != HEXIR_OK)
          return st;
        buffers[i] = args[i]->dev[0];
      }
      Span *span = begin_span(cuda[0]);
      hexir_status_t st = cuda[0]->launch(
          exe_base + exe.image_offset, exe.image_size, exe.name, exe.grid_x,
          exe.grid_y, exe.block_x, exe.block_y, buffers,
          static_cast<unsigned>(argc));
      end_span(span);
      if (st == HEXIR_OK)
        written_on_device(*args[argc - 1], 0);
      return st;
    }

    // cpu placement.
    if (exe.image_size)
      return HEXIR_ERROR_UNIMPLEMENTED;  // no host images exist
    hexir_status_t st = check_sizes(exe, args, argc);
    if (st != HEXIR_OK)
      return st;
    if (trace)
      std::fprintf(stderr, "hexir: dispatch %.32s %s %ux%ux%u on cpu\n", exe.name,
                   hexir_kernel_kind_string(exe.kind), exe.m, exe.n, exe.k);
    return run_host(exe, args);
  }

  hexir_status_t print(uint64_t index, uint64_t rows, uint64_t cols) {
    Slot *s = slot(index);
    if (!s)
      return HEXIR_ERROR_INVALID_MODULE;
    if (rows != 0 && cols > UINT64_MAX / 8 / rows)
      return HEXIR_ERROR_INVALID_MODULE;
    if (rows * cols * 8 > s->bytes)
      return HEXIR_ERROR_INVALID_MODULE;
    const uint8_t *data = nullptr;
    hexir_status_t st = on_host(*s, &data);
    if (st != HEXIR_OK)
      return st;
    const double *v = reinterpret_cast<const double *>(data);
    for (uint64_t i = 0; i < rows; ++i) {
      for (uint64_t j = 0; j < cols; ++j)
        std::printf("%f ", v[i * cols + j]);
      std::printf("\n");
    }
    return HEXIR_OK;
  }

  // Wait for every GPU, collect kernel error words and span timings.
  // Page-locked host memory (registered or allocated by the driver)?
  bool page_locked(const void *p) {
    if (cuda.empty())
      return false;
    ContextGuard guard(cuda.front()->state->context);
    unsigned int type = 0;
    return driver().PointerGetAttribute(
               &type, CU_POINTER_ATTRIBUTE_MEMORY_TYPE,
               reinterpret_cast<CUdeviceptr>(p)) == CUDA_SUCCESS &&
           type == CU_MEMORYTYPE_HOST;
  }

  // Large captures into pageable memory go through a page-locked block.
  void stage_capture(void *out, size_t size) {
    capture_out = out;
    capture_size = size;
    constexpr size_t kStageMinBytes = 1u << 20;
    if (cuda.empty() || size < kStageMinBytes || page_locked(out))
      return;
    void *stage = pinned_take(size, cuda.front()->state->context);
    if (!stage)
      return;  // the downloads go to `out` directly, at pageable speed
    pinned.emplace_back(stage, size);
    capture_user = out;
    capture_out = stage;
  }

  // Streamed chunks of the capture, each copied to the caller's memory once
  // its download has landed (the later ones may still be computing).
  hexir_status_t drain_staged() {
    const Driver &d = driver();
    hexir_status_t st = HEXIR_OK;
    for (auto &chunk : staged_chunks) {
      const uint64_t off = std::get<0>(chunk), bytes = std::get<1>(chunk);
      CUevent ev = std::get<2>(chunk);
      ContextGuard guard(cuda.front()->state->context);
      if (d.EventSynchronize(ev) != CUDA_SUCCESS)
        st = HEXIR_ERROR_DEVICE;
      else if (st == HEXIR_OK)
        parallel_copy(static_cast<uint8_t *>(capture_user) + off,
                      static_cast<const uint8_t *>(capture_out) + off, bytes);
      d.EventDestroy(ev);
      staged_copied += bytes;
    }
    staged_chunks.clear();
    return st;
  }

  hexir_status_t settle() {
    hexir_status_t result = HEXIR_OK;
    for (CudaDevice *dev : cuda) {
      std::string error;
      if (check_device(dev->state, dev->stream, &error) != HEXIR_OK) {
        report(error);
        result = HEXIR_ERROR_DEVICE;
      }
    }
    double ms = 0.0;
    for (Span &sp : spans) {
      ContextGuard g(sp.device->state->context);
      float t = 0.0f;
      if (driver().EventElapsedTime(&t, sp.start, sp.stop) == CUDA_SUCCESS)
        ms += t;
    }
    g_last_kernel_ms = ms;
    return result;
  }

  hexir_status_t capture(uint64_t index, void *out, size_t size) {
    Slot *s = slot(index);
    if (!s || size > s->bytes)
      return HEXIR_ERROR_INVALID_ARGUMENT;
    if (!s->host_valid && !s->rodata && !s->zero && !s->dev_valid.empty()) {
      const int p = *s->dev_valid.begin();
      return hexir_buffer_read(s->dev[p], out, size);
    }
    const uint8_t *data = nullptr;
    hexir_status_t st = on_host(*s, &data);
    if (st == HEXIR_OK && size)
      std::memcpy(out, data, size);
    return st;
  }
};

hexir_status_t execute_unguarded(const hexir_module_t *module,
                                 hexir_device_t *primary,
                                 std::vector<CudaDevice *> cuda,
                                 const char *entry, void *out_result,
                                 size_t out_size);

// Sizes in a module are untrusted: a host buffer they ask for may not exist.
// No C++ exception crosses the C ABI.
hexir_status_t execute(const hexir_module_t *module, hexir_device_t *primary,
                       std::vector<CudaDevice *> cuda, const char *entry,
                       void *out_result, size_t out_size) {
  try {
    return execute_unguarded(module, primary, std::move(cuda), entry,
                             out_result, out_size);
  } catch (const std::bad_alloc &) {
    report("host allocation failed while executing the module");
    return HEXIR_ERROR_OUT_OF_MEMORY;
  } catch (const std::exception &e) {
    report(std::string("execute failed: ") + e.what());
    return HEXIR_ERROR_INVALID_MODULE;
  }
}

hexir_status_t execute_unguarded(const hexir_module_t *module,
                                 hexir_device_t *primary,
                                 std::vector<CudaDevice *> cuda,
                                 const char *entry, void *out_result,
                                 size_t out_size) {
  if (!module || !entry)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  g_last_kernel_ms = 0.0;
  const void *symbols_data = nullptr, *program_data = nullptr;
  uint64_t symbols_size = 0, program_size = 0;
  if (hexir_module_section(module, HEXIR_SECTION_SYMBOLS, &symbols_data,
                           &symbols_size) != HEXIR_OK ||
      hexir_module_section(module, HEXIR_SECTION_PROGRAM, &program_data,
                           &program_size) != HEXIR_OK)
    return HEXIR_ERROR_INVALID_MODULE;

  auto vm = std::make_unique<Vm>();
  vm->module = module;
  vm->primary = primary;
  vm->cuda = std::move(cuda);
  const char *trace = std::getenv("HEXIR_TRACE");
  vm->trace = trace && trace[0] && trace[0] != '0';

  const void *data = nullptr;
  uint64_t size = 0;
  if (hexir_module_section(module, HEXIR_SECTION_RODATA, &data, &size) ==
      HEXIR_OK) {
    vm->rodata = static_cast<const uint8_t *>(data);
    vm->rodata_size = size;
  }
  if (hexir_module_section(module, HEXIR_SECTION_EXECUTABLES, &data, &size) ==
          HEXIR_OK &&
      size >= sizeof(hexir_executable_header_t)) {
    hexir_executable_header_t header;
    std::memcpy(&header, data, sizeof(header));
    const uint64_t table = sizeof(header) + static_cast<uint64_t>(header.count) *
                                                sizeof(hexir_executable_entry_t);
    if (table > size)
      return HEXIR_ERROR_INVALID_MODULE;
    vm->exes = reinterpret_cast<const hexir_executable_entry_t *>(
        static_cast<const uint8_t *>(data) + sizeof(header));
    vm->exe_count = header.count;
    vm->exe_base = static_cast<const uint8_t *>(data);
    vm->exe_size = size;
  }
  if (hexir_module_section(module, HEXIR_SECTION_LAUNCH, &data, &size) ==
          HEXIR_OK &&
      size >= sizeof(hexir_launch_header_t)) {
    hexir_launch_header_t header;
    std::memcpy(&header, data, sizeof(header));
    const uint64_t table = sizeof(header) + static_cast<uint64_t>(header.count) *
                                                sizeof(hexir_launch_entry_t);
    if (table > size)
      return HEXIR_ERROR_INVALID_MODULE;
    vm->launches = reinterpret_cast<const hexir_launch_entry_t *>(
        static_cast<const uint8_t *>(data) + sizeof(header));
    vm->launch_count = header.count;
  }

  const auto *symbols = static_cast<const hexir_symbol_entry_t *>(symbols_data);
  const uint64_t symbol_count = symbols_size / sizeof(hexir_symbol_entry_t);
  uint64_t pc = 0;
  bool found = false;
  for (uint64_t i = 0; i < symbol_count; ++i) {
    if (std::strncmp(symbols[i].name, entry, HEXIR_NAME_SIZE) == 0) {
      pc = symbols[i].program_offset;
      found = true;
      break;
    }
  }
  if (!found)
    return HEXIR_ERROR_NOT_FOUND;

  const uint8_t *program = static_cast<const uint8_t *>(program_data);
  vm->program = program;
  vm->program_size = program_size;
  // Find the entry's last DISPATCH: its destination is what a capture copies
  // out, so that dispatch may stream its result straight to out_result.
  if (out_result && out_size) {
    uint64_t scan = pc;
    while (scan + sizeof(hexir_command_header_t) <= program_size) {
      hexir_command_header_t h;
      std::memcpy(&h, program + scan, sizeof(h));
      const uint64_t next = scan + sizeof(h) + static_cast<uint64_t>(h.operand_count) * 8;
      if (next > program_size)
        break;
      if (h.kind == HEXIR_CMD_DISPATCH)
        vm->last_dispatch_pc = scan;
      if (h.kind == HEXIR_CMD_END)
        break;
      scan = next;
    }
    vm->stage_capture(out_result, out_size);
  }
  hexir_status_t status = HEXIR_OK;
  int64_t result_slot = -1;
  while (status == HEXIR_OK) {
    vm->current_pc = pc;
    if (pc + sizeof(hexir_command_header_t) > program_size) {
      status = HEXIR_ERROR_INVALID_MODULE;
      break;
    }
    hexir_command_header_t header;
    std::memcpy(&header, program + pc, sizeof(header));
    pc += sizeof(header);
    const uint64_t operand_bytes =
        static_cast<uint64_t>(header.operand_count) * sizeof(uint64_t);
    if (pc + operand_bytes > program_size) {
      status = HEXIR_ERROR_INVALID_MODULE;
      break;
    }
    std::vector<uint64_t> ops(header.operand_count);
    if (operand_bytes)
      std::memcpy(ops.data(), program + pc, operand_bytes);
    pc += operand_bytes;

    switch (header.kind) {
    case HEXIR_CMD_END: {
      hexir_status_t drained = vm->drain_staged();
      hexir_status_t settled = vm->settle();
      if (settled != HEXIR_OK)
        return settled;
      if (drained != HEXIR_OK)
        return drained;
      if (out_result && out_size && result_slot >= 0 && !vm->capture_done) {
        status = vm->capture(static_cast<uint64_t>(result_slot),
                             vm->capture_out, out_size);
        if (status == HEXIR_OK && vm->capture_user)
          parallel_copy(vm->capture_user, vm->capture_out, out_size);
      }
      return status;
    }
    case HEXIR_CMD_ALLOC:
      if (header.operand_count != 2) {
        status = HEXIR_ERROR_INVALID_MODULE;
        break;
      }
      status = vm->bind(ops[0], ops[1]);
      if (status == HEXIR_OK)
        vm->slots[ops[0]].zero = true;
      break;
    case HEXIR_CMD_CONST: {
      if (header.operand_count != 3) {
        status = HEXIR_ERROR_INVALID_MODULE;
        break;
      }
      const uint64_t offset = ops[1], bytes = ops[2];
      if (offset > vm->rodata_size || bytes > vm->rodata_size - offset) {
        status = HEXIR_ERROR_INVALID_MODULE;
        break;
      }
      status = vm->bind(ops[0], bytes);
      if (status == HEXIR_OK) {
        vm->slots[ops[0]].rodata = vm->rodata + offset;
        status = vm->adopt_prefetched(vm->slots[ops[0]], offset);
      }
      break;
    }
    case HEXIR_CMD_DISPATCH:
      status = vm->dispatch(ops.data(), header.operand_count);
      if (status == HEXIR_OK && header.operand_count >= 3)
        result_slot = static_cast<int64_t>(ops[header.operand_count - 1]);
      if (status == HEXIR_OK)
        status = vm->prefetch_ahead(pc);
      break;
    case HEXIR_CMD_PRINT:
      if (header.operand_count != 3)
        status = HEXIR_ERROR_INVALID_MODULE;
      else
        status = vm->print(ops[0], ops[1], ops[2]);
      break;
    default:
      status = HEXIR_ERROR_INVALID_MODULE;
      break;
    }
  }
  vm->settle();
  return status;
}

}  // namespace

}  // namespace hexir

using namespace hexir;

extern "C" {

const char *hexir_kernel_kind_string(uint32_t kind) {
  switch (kind) {
  case HEXIR_KERNEL_MATMUL: return "matmul";
  case HEXIR_KERNEL_ADD: return "add";
  case HEXIR_KERNEL_RELU: return "relu";
  case HEXIR_KERNEL_MATMUL_RELU: return "matmul_relu";
  case HEXIR_KERNEL_MATMUL_ADD: return "matmul_add";
  case HEXIR_KERNEL_MATMUL_ADD_RELU: return "matmul_add_relu";
  case HEXIR_KERNEL_LEAKY_RELU: return "leaky_relu";
  case HEXIR_KERNEL_ELU: return "elu";
  case HEXIR_KERNEL_SIGMOID: return "sigmoid";
  case HEXIR_KERNEL_TANH: return "tanh";
  case HEXIR_KERNEL_SOFTMAX: return "softmax";
  case HEXIR_KERNEL_GELU: return "gelu";
  case HEXIR_KERNEL_SWISH: return "swish";
  case HEXIR_KERNEL_MISH: return "mish";
  }
  return "unknown";
}

hexir_status_t hexir_execute(const hexir_module_t *module,
                             hexir_device_t *device, const char *entry) {
  return hexir_execute_capture(module, device, entry, nullptr, 0);
}

hexir_status_t hexir_execute_capture(const hexir_module_t *module,
                                     hexir_device_t *device, const char *entry,
                                     void *out_result, size_t out_size) {
  if (!module || !device || !entry)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  std::vector<CudaDevice *> cuda;
  if (CudaDevice *c = as_cuda(device))
    cuda.push_back(c);
  return execute(module, device, std::move(cuda), entry, out_result, out_size);
}

hexir_status_t hexir_execute_devices(const hexir_module_t *module,
                                     hexir_device_t *const *devices,
                                     unsigned device_count, const char *entry,
                                     void *out_result, size_t out_size) {
  if (!module || !entry || (device_count && !devices))
    return HEXIR_ERROR_INVALID_ARGUMENT;
  std::vector<CudaDevice *> cuda;
  for (unsigned i = 0; i < device_count; ++i) {
    CudaDevice *c = as_cuda(devices[i]);
    if (!c)
      return HEXIR_ERROR_INVALID_ARGUMENT;
    cuda.push_back(c);
  }
  hexir_device_t *primary = device_count ? devices[0] : nullptr;
  static hexir_device_t *host_only = nullptr;
  if (!primary) {
    if (!host_only && hexir_device_create(HEXIR_DEVICE_CPU, &host_only) != HEXIR_OK)
      return HEXIR_ERROR_OUT_OF_MEMORY;
    primary = host_only;
  }
  return execute(module, primary, std::move(cuda), entry, out_result, out_size);
}

double hexir_last_execute_kernel_ms(void) { return g_last_kernel_ms; }

hexir_status_t hexir_module_keep_constants(hexir_module_t *module, int enable) {
  if (!module)
    return HEXIR_ERROR_INVALID_ARGUMENT;
  ModuleState *ms = module_state(module);
  if (!ms)
    return HEXIR_ERROR_OUT_OF_MEMORY;
  std::lock_guard<std::mutex> lock(ms->mu);
  ms->keep_constants.store(enable != 0);
  if (!enable)
    ms->drop_resident();
  return HEXIR_OK;
}

size_t hexir_module_kept_bytes(const hexir_module_t *module) {
  ModuleState *ms = module_state(module);
  if (!ms)
    return 0;
  std::lock_guard<std::mutex> lock(ms->mu);
  size_t total = 0;
  for (const ResidentConst &rc : ms->resident)
    total += rc.bytes;
  return total;
}

}  // extern "C"
