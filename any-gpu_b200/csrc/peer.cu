// Peer memory between the processes of one node (one process per GPU):
// CUDA IPC handles of device memory and of events, and stream-ordered copies
// into a peer's memory.  A sharded job all-gathers its outputs with these on
// the copy engines: every rank pushes each finished round of its results
// straight into the same slot of every peer's output buffer over NVLink,
// using no SMs, so the pushes run beside the next round's kernels (NCCL's
// gather kernels need SMs, which the persistent contraction kernels hold).
//
// Completion crosses processes either through interprocess events (a rank
// records its event after its pushes; a peer's stream waits on it once the
// host side knows the record was issued) or through flag words in device
// memory: after its pushes a rank's stream stores the step number into every
// peer's flag (signal_peers_kernel, a system-scope release), and each rank's
// stream waits until all its flags reach the step (wait_flags_kernel, a
// bounded spin: on expiry it records a code in the device status word, which
// the next agpu_synchronize reports as AGPU_ERR_TIMEOUT, and returns).
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "agpu_internal.cuh"

using namespace agpu;

namespace {

static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(agpu_ipc_handle), "IPC handle size");
static_assert(sizeof(cudaIpcEventHandle_t) == sizeof(agpu_ipc_handle), "IPC handle size");

// cuMemGetAddressRange through the runtime's driver entry point, so that the
// library links no driver symbol directly (it loads where libcuda is absent).
using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(p);
  });
  return fn;
}

agpu_status select(agpu_device* dev, const char* fn) {
  if (!dev) return fail(AGPU_ERR_INVALID, "%s: NULL device", fn);
  AGPU_CUDA(cudaSetDevice(dev->ordinal));
  return AGPU_OK;
}

constexpr int kMaxPeers = 16;

struct PeerFlags {
  unsigned int* p[kMaxPeers];
};

// Store `value` into each peer's flag word (system-scope release: every write
// this stream made before -- the copies of the data -- is complete first).
__global__ void signal_peers_kernel(PeerFlags flags, int count, unsigned int value) {
  const int i = threadIdx.x;
  if (i < count)
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flags.p[i]), "r"(value) : "memory");
}

// One warp: wait until flags[i] >= target (wrapping compare) for every i <
// count, each read an acquire at system scope; give up after limit_ns of
// global time, record `code` in the status word and return.
__global__ void wait_flags_kernel(const unsigned int* flags, int count, unsigned int target,
                                  unsigned long long limit_ns, unsigned int* status,
                                  unsigned int code) {
  const int lane = threadIdx.x;
  unsigned long long t0 = 0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (uint32_t it = 0;; ++it) {
    bool done = true;
    if (lane < count) {
      unsigned int v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + lane) : "memory");
      done = (int)(v - target) >= 0;
    }
    if (__all_sync(0xffffffffu, done)) return;
    if ((it & 63u) == 63u) {
      unsigned long long t1;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
      if (t1 - t0 > limit_ns) {
        if (lane == 0) atomicCAS(status, 0u, code);
        return;
      }
    }
  }
}

}  // namespace

extern "C" {

agpu_status agpu_signal_peers(agpu_device* dev, unsigned int* const* peer_flags, uint32_t count,
                              uint32_t value, void* stream) {
  AGPU_TRY(select(dev, "agpu_signal_peers"));
  if (count == 0) return AGPU_OK;
  if (!peer_flags || count > kMaxPeers)
    return fail(AGPU_ERR_INVALID, "agpu_signal_peers: %u flags (at most %d)", count, kMaxPeers);
  PeerFlags f = {};
  for (uint32_t i = 0; i < count; ++i) {
    if (!peer_flags[i]) return fail(AGPU_ERR_INVALID, "agpu_signal_peers: NULL flag %u", i);
    f.p[i] = peer_flags[i];
  }
  signal_peers_kernel<<<1, 32, 0, pick_stream(dev, stream)>>>(f, (int)count, value);
  return after_launch(dev, "signal_peers_kernel");
}

agpu_status agpu_wait_flags(agpu_device* dev, const unsigned int* flags, uint32_t count,
                            uint32_t target, uint32_t limit_us, void* stream) {
  AGPU_TRY(select(dev, "agpu_wait_flags"));
  if (count == 0) return AGPU_OK;
  if (!flags || count > 32 || limit_us == 0 || limit_us > 10000000u)
    return fail(AGPU_ERR_INVALID, "agpu_wait_flags: %u flags (at most 32), limit %u us", count,
                limit_us);
  wait_flags_kernel<<<1, 32, 0, pick_stream(dev, stream)>>>(flags, (int)count, target,
                                                            1000ull * limit_us, dev->d_status,
                                                            AGPU_WAIT_FLAGS_CODE);
  return after_launch(dev, "wait_flags_kernel");
}

agpu_status agpu_ipc_export(agpu_device* dev, const void* dptr, agpu_ipc_handle* handle,
                            uint64_t* offset) {
  AGPU_TRY(select(dev, "agpu_ipc_export"));
  if (!dptr || !handle || !offset) return fail(AGPU_ERR_INVALID, "agpu_ipc_export: NULL argument");
  // IPC handles name whole allocations: export the one holding dptr
  AddressRangeFn range = address_range_fn();
  if (!range) return fail(AGPU_ERR_CUDA, "agpu_ipc_export: cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(dptr));
  if (r != CUDA_SUCCESS)
    return fail(AGPU_ERR_INVALID, "agpu_ipc_export: %p is not device memory (%d)", dptr, (int)r);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(AGPU_ERR_UNSUPPORTED,
                "agpu_ipc_export: allocation at %p cannot be shared (%s); it must come from "
                "cudaMalloc", reinterpret_cast<void*>(base), cudaGetErrorString(e));
  }
  std::memcpy(handle->bytes, &h, sizeof(h));
  *offset = reinterpret_cast<CUdeviceptr>(dptr) - base;
  return AGPU_OK;
}

agpu_status agpu_ipc_import(agpu_device* dev, const agpu_ipc_handle* handle, void** base) {
  AGPU_TRY(select(dev, "agpu_ipc_import"));
  if (!handle || !base) return fail(AGPU_ERR_INVALID, "agpu_ipc_import: NULL argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  *base = nullptr;
  AGPU_CUDA(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess));
  return AGPU_OK;
}

agpu_status agpu_ipc_close(agpu_device* dev, void* base) {
  AGPU_TRY(select(dev, "agpu_ipc_close"));
  if (!base) return AGPU_OK;
  AGPU_CUDA(cudaIpcCloseMemHandle(base));
  return AGPU_OK;
}

agpu_status agpu_ipc_event_create(agpu_device* dev, void** event, agpu_ipc_handle* handle) {
  AGPU_TRY(select(dev, "agpu_ipc_event_create"));
  if (!event || !handle) return fail(AGPU_ERR_INVALID, "agpu_ipc_event_create: NULL argument");
  cudaEvent_t e = nullptr;
  AGPU_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming | cudaEventInterprocess));
  cudaIpcEventHandle_t h;
  const cudaError_t err = cudaIpcGetEventHandle(&h, e);
  if (err != cudaSuccess) {
    cudaEventDestroy(e);
    return cuda_status(err, "agpu_ipc_event_create: cudaIpcGetEventHandle");
  }
  std::memcpy(handle->bytes, &h, sizeof(h));
  *event = e;
  return AGPU_OK;
}

agpu_status agpu_ipc_event_import(agpu_device* dev, const agpu_ipc_handle* handle, void** event) {
  AGPU_TRY(select(dev, "agpu_ipc_event_import"));
  if (!handle || !event) return fail(AGPU_ERR_INVALID, "agpu_ipc_event_import: NULL argument");
  cudaIpcEventHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  cudaEvent_t e = nullptr;
  AGPU_CUDA(cudaIpcOpenEventHandle(&e, h));
  *event = e;
  return AGPU_OK;
}

agpu_status agpu_event_destroy(agpu_device* dev, void* event) {
  AGPU_TRY(select(dev, "agpu_event_destroy"));
  if (event) AGPU_CUDA(cudaEventDestroy(static_cast<cudaEvent_t>(event)));
  return AGPU_OK;
}

agpu_status agpu_event_record(agpu_device* dev, void* event, void* stream) {
  AGPU_TRY(select(dev, "agpu_event_record"));
  if (!event) return fail(AGPU_ERR_INVALID, "agpu_event_record: NULL event");
  AGPU_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(event), pick_stream(dev, stream)));
  return AGPU_OK;
}

agpu_status agpu_stream_wait_event(agpu_device* dev, void* stream, void* event) {
  AGPU_TRY(select(dev, "agpu_stream_wait_event"));
  if (!event) return fail(AGPU_ERR_INVALID, "agpu_stream_wait_event: NULL event");
  AGPU_CUDA(cudaStreamWaitEvent(pick_stream(dev, stream), static_cast<cudaEvent_t>(event), 0));
  return AGPU_OK;
}

agpu_status agpu_copy_async(agpu_device* dev, void* dst, const void* src, uint64_t bytes,
                            void* stream) {
  AGPU_TRY(select(dev, "agpu_copy_async"));
  if (bytes == 0) return AGPU_OK;
  if (!dst || !src) return fail(AGPU_ERR_INVALID, "agpu_copy_async: NULL pointer");
  AGPU_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, pick_stream(dev, stream)));
  return AGPU_OK;
}

}  // extern "C"
