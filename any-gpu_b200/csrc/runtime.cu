// Device runtime behind the C ABI: device handle, stream, stream-ordered
// memory pool, buffers, H2D/D2H, error reporting.
//
// Replaces the wgpu plumbing of the reference's src/device.rs:12-190
// (instance/adapter/queue, create_buffer_init, map_async read-back and the
// WGSL pipeline cache).  CUDA modules are loaded once with the library, so
// there is no per-shader compile step to cache.
#include <cstdarg>
#include <cstring>

#include "agpu_internal.cuh"
#include "ptx.cuh"

namespace agpu {

static thread_local char g_err[1024] = {0};
thread_local int g_thread_precision = -1;

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

agpu_status fail(agpu_status s, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return s;
}

agpu_status cuda_status(cudaError_t e, const char* what) {
  set_error("%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
  if (e == cudaErrorMemoryAllocation) return AGPU_ERR_OOM;
  if (e == cudaErrorNoDevice || e == cudaErrorInvalidDevice) return AGPU_ERR_NO_DEVICE;
  return AGPU_ERR_CUDA;
}

agpu_status pool_alloc(agpu_device* dev, size_t bytes, void** out, cudaStream_t s) {
  *out = nullptr;
  if (bytes == 0) bytes = 256;  // keep every buffer addressable
  cudaError_t e = cudaMallocFromPoolAsync(out, bytes, dev->pool, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(AGPU_ERR_OOM, "device pool: cannot allocate %zu bytes (%s)", bytes,
                cudaGetErrorString(e));
  }
  return AGPU_OK;
}

void pool_free(agpu_device* dev, void* p, cudaStream_t s) {
  (void)dev;
  if (p) cudaFreeAsync(p, s);
}

agpu_status new_buffer(agpu_device* dev, uint64_t n, agpu_buffer** out) {
  void* p = nullptr;
  AGPU_TRY(pool_alloc(dev, n * sizeof(float), &p, dev->stream));
  auto* b = new agpu_buffer;
  b->dptr = static_cast<float*>(p);
  b->len = n;
  b->dev = dev;
  dev->refs.fetch_add(1, std::memory_order_relaxed);
  *out = b;
  return AGPU_OK;
}

void device_release(agpu_device* dev) {
  if (dev->refs.fetch_sub(1, std::memory_order_acq_rel) != 1) return;
  cudaSetDevice(dev->ordinal);
  cudaStreamSynchronize(dev->stream);
  cudaFree(dev->d_status);
  cudaStreamDestroy(dev->stream);
  if (dev->aux) {
    cudaStreamSynchronize(dev->aux);
    cudaStreamDestroy(dev->aux);
  }
  // Blocks still out (scratch freed on a caller stream that has not reached
  // the free yet) keep the pool alive until they come back.
  if (dev->pool) cudaMemPoolDestroy(dev->pool);
  delete dev;
}

cudaStream_t aux_stream(agpu_device* dev) {
  std::lock_guard<std::mutex> lock(dev->mu);
  if (!dev->aux && cudaStreamCreateWithFlags(&dev->aux, cudaStreamNonBlocking) != cudaSuccess) {
    cudaGetLastError();
    dev->aux = nullptr;
  }
  return dev->aux;
}

agpu_status after_launch(agpu_device* dev, const char* kernel, int n_launches) {
  dev->launches.fetch_add(n_launches, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, kernel);
  return AGPU_OK;
}

agpu_status check_device_status(agpu_device* dev) {
  unsigned int h = 0;
  AGPU_CUDA(cudaMemcpyAsync(&h, dev->d_status, sizeof(h), cudaMemcpyDeviceToHost, dev->stream));
  AGPU_CUDA(cudaStreamSynchronize(dev->stream));
  if (h != 0) {
    AGPU_CUDA(cudaMemsetAsync(dev->d_status, 0, sizeof(unsigned int), dev->stream));
    return fail(AGPU_ERR_TIMEOUT, "a device-side bounded wait expired (code 0x%x)", h);
  }
  return AGPU_OK;
}

// Failure-path self-test: one warp waits on an mbarrier that no thread ever
// arrives on.  The wait gives up after limit_ns, records `code` in the device
// status word and the kernel returns: the path every pipeline wait of the
// contraction kernels takes when its producer never arrives, exercised
// without TMA, tensor cores or tensor memory.
__global__ void wait_timeout_selftest_kernel(unsigned int* status, unsigned long long limit_ns,
                                             unsigned int code) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    ptx::mbar_init(&bar, 1);
    abort_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();
  ptx::mbar_wait_for(&bar, 0, status, code, &abort_flag, limit_ns);
  __syncthreads();
}

}  // namespace agpu

using namespace agpu;

extern "C" {

const char* agpu_last_error_message(void) { return agpu::g_err; }

const char* agpu_status_string(agpu_status s) {
  switch (s) {
    case AGPU_OK: return "ok";
    case AGPU_ERR_SHAPE: return "shape mismatch";
    case AGPU_ERR_INVALID: return "invalid argument";
    case AGPU_ERR_CUDA: return "cuda error";
    case AGPU_ERR_OOM: return "out of device memory";
    case AGPU_ERR_NO_DEVICE: return "no such device";
    case AGPU_ERR_TIMEOUT: return "device wait timed out";
    case AGPU_ERR_UNSUPPORTED: return "unsupported";
  }
  return "unknown status";
}

agpu_status agpu_device_create(int ordinal, agpu_device** out) {
  if (!out) return fail(AGPU_ERR_INVALID, "agpu_device_create: out is NULL");
  *out = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    cudaGetLastError();
    return fail(AGPU_ERR_NO_DEVICE, "no CUDA device available (%s)", cudaGetErrorString(e));
  }
  if (ordinal < 0 || ordinal >= count)
    return fail(AGPU_ERR_NO_DEVICE, "device ordinal %d out of range [0,%d)", ordinal, count);
  AGPU_CUDA(cudaSetDevice(ordinal));
  cudaDeviceProp prop;
  AGPU_CUDA(cudaGetDeviceProperties(&prop, ordinal));
  if (prop.major != 10)
    return fail(AGPU_ERR_UNSUPPORTED, "device %d (%s) is sm_%d%d; this library is built for sm_100a",
                ordinal, prop.name, prop.major, prop.minor);
  auto* d = new agpu_device;
  d->ordinal = ordinal;
  d->sm_count = prop.multiProcessorCount;
  snprintf(d->name, sizeof(d->name), "%s", prop.name);
  e = cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) { delete d; return cuda_status(e, "cudaStreamCreate"); }
  // A pool of this handle's own (not the device's default pool, which other
  // libraries in the process, torch's async allocator among them, share):
  // freed blocks stay cached in it instead of going back to the driver at
  // every synchronisation, so steady-state ops never reach cudaMalloc, and
  // no other pool user sees that setting.
  cudaMemPoolProps props = {};
  props.allocType = cudaMemAllocationTypePinned;
  props.handleTypes = cudaMemHandleTypeNone;
  props.location.type = cudaMemLocationTypeDevice;
  props.location.id = ordinal;
  e = cudaMemPoolCreate(&d->pool, &props);
  if (e != cudaSuccess) {
    cudaStreamDestroy(d->stream);
    delete d;
    return cuda_status(e, "cudaMemPoolCreate");
  }
  uint64_t threshold = UINT64_MAX;
  cudaMemPoolSetAttribute(d->pool, cudaMemPoolAttrReleaseThreshold, &threshold);
  e = cudaMalloc(&d->d_status, sizeof(unsigned int));
  if (e != cudaSuccess) {
    cudaMemPoolDestroy(d->pool);
    cudaStreamDestroy(d->stream);
    delete d;
    return cuda_status(e, "cudaMalloc(status)");
  }
  cudaMemset(d->d_status, 0, sizeof(unsigned int));
  *out = d;
  return AGPU_OK;
}

agpu_status agpu_device_destroy(agpu_device* dev) {
  if (!dev) return AGPU_OK;
  cudaSetDevice(dev->ordinal);
  cudaStreamSynchronize(dev->stream);
  device_release(dev);
  return AGPU_OK;
}

agpu_status agpu_device_name(const agpu_device* dev, char* buf, size_t n) {
  if (!dev || !buf || n == 0) return fail(AGPU_ERR_INVALID, "agpu_device_name: bad argument");
  snprintf(buf, n, "%s", dev->name);
  return AGPU_OK;
}

agpu_status agpu_device_sm_count(const agpu_device* dev, int* out) {
  if (!dev || !out) return fail(AGPU_ERR_INVALID, "agpu_device_sm_count: bad argument");
  *out = dev->sm_count;
  return AGPU_OK;
}

agpu_status agpu_device_ordinal(const agpu_device* dev, int* out) {
  if (!dev || !out) return fail(AGPU_ERR_INVALID, "agpu_device_ordinal: bad argument");
  *out = dev->ordinal;
  return AGPU_OK;
}

void* agpu_device_stream(const agpu_device* dev) { return dev ? (void*)dev->stream : nullptr; }

agpu_status agpu_synchronize(agpu_device* dev) {
  if (!dev) return fail(AGPU_ERR_INVALID, "agpu_synchronize: NULL device");
  AGPU_CUDA(cudaStreamSynchronize(dev->stream));
  return check_device_status(dev);
}

agpu_status agpu_set_precision(agpu_device* dev, agpu_precision p) {
  if (!dev) return fail(AGPU_ERR_INVALID, "agpu_set_precision: NULL device");
  if (p != AGPU_PREC_TF32 && p != AGPU_PREC_TF32X3 && p != AGPU_PREC_FFMA)
    return fail(AGPU_ERR_INVALID, "agpu_set_precision: unknown mode %d", (int)p);
  dev->precision.store(p, std::memory_order_relaxed);
  return AGPU_OK;
}

agpu_status agpu_get_precision(const agpu_device* dev, agpu_precision* p) {
  if (!dev || !p) return fail(AGPU_ERR_INVALID, "agpu_get_precision: bad argument");
  *p = static_cast<agpu_precision>(dev->precision.load(std::memory_order_relaxed));
  return AGPU_OK;
}

agpu_status agpu_set_thread_precision(int mode) {
  if (mode != -1 && mode != AGPU_PREC_TF32 && mode != AGPU_PREC_TF32X3 && mode != AGPU_PREC_FFMA)
    return fail(AGPU_ERR_INVALID, "agpu_set_thread_precision: unknown mode %d", mode);
  g_thread_precision = mode;
  return AGPU_OK;
}

int agpu_get_thread_precision(void) { return g_thread_precision; }

uint64_t agpu_device_launch_count(const agpu_device* dev) {
  return dev ? dev->launches.load() : 0;
}

agpu_status agpu_upload(agpu_device* dev, const float* host, uint64_t n, agpu_buffer** out) {
  if (!dev || !out || (!host && n)) return fail(AGPU_ERR_INVALID, "agpu_upload: bad argument");
  AGPU_CUDA(cudaSetDevice(dev->ordinal));
  AGPU_TRY(new_buffer(dev, n, out));
  if (n) {
    cudaError_t e = cudaMemcpyAsync((*out)->dptr, host, n * sizeof(float),
                                    cudaMemcpyHostToDevice, dev->stream);
    if (e != cudaSuccess) {
      agpu_buffer_free(*out);
      *out = nullptr;
      return cuda_status(e, "agpu_upload");
    }
  }
  return AGPU_OK;
}

// Zero-filled, as the reference's wgpu buffers are (src/device.rs:97-112).
agpu_status agpu_alloc(agpu_device* dev, uint64_t n, agpu_buffer** out) {
  if (!dev || !out) return fail(AGPU_ERR_INVALID, "agpu_alloc: bad argument");
  AGPU_CUDA(cudaSetDevice(dev->ordinal));
  AGPU_TRY(new_buffer(dev, n, out));
  if (n) {
    const cudaError_t e = cudaMemsetAsync((*out)->dptr, 0, n * sizeof(float), dev->stream);
    if (e != cudaSuccess) {
      agpu_buffer_free(*out);
      *out = nullptr;
      return cuda_status(e, "agpu_alloc: zero fill");
    }
  }
  return AGPU_OK;
}

agpu_status agpu_write(agpu_device* dev, agpu_buffer* buf, const float* host, uint64_t n) {
  if (!dev || !buf || (!host && n)) return fail(AGPU_ERR_INVALID, "agpu_write: bad argument");
  if (n != buf->len)
    return fail(AGPU_ERR_SHAPE, "agpu_write: buffer has %llu elems, host has %llu",
                (unsigned long long)buf->len, (unsigned long long)n);
  AGPU_CUDA(cudaSetDevice(dev->ordinal));
  AGPU_CUDA(cudaMemcpyAsync(buf->dptr, host, n * sizeof(float), cudaMemcpyHostToDevice,
                            dev->stream));
  return AGPU_OK;
}

agpu_status agpu_read(agpu_device* dev, const agpu_buffer* buf, float* host, uint64_t n) {
  if (!dev || !buf || (!host && n)) return fail(AGPU_ERR_INVALID, "agpu_read: bad argument");
  if (n != buf->len)
    return fail(AGPU_ERR_SHAPE, "agpu_read: buffer has %llu elems, host has %llu",
                (unsigned long long)buf->len, (unsigned long long)n);
  AGPU_CUDA(cudaSetDevice(dev->ordinal));
  if (n)
    AGPU_CUDA(cudaMemcpyAsync(host, buf->dptr, n * sizeof(float), cudaMemcpyDeviceToHost,
                              dev->stream));
  AGPU_CUDA(cudaStreamSynchronize(dev->stream));
  return check_device_status(dev);
}

static agpu_status copy_async(agpu_device* dev, const agpu_buffer* buf, uint64_t offset,
                              uint64_t n, const void* host, bool to_device, void* stream,
                              const char* fn) {
  if (!dev || !buf || (!host && n)) return fail(AGPU_ERR_INVALID, "%s: bad argument", fn);
  if (offset > buf->len || n > buf->len - offset)
    return fail(AGPU_ERR_SHAPE, "%s: elements [%llu, %llu) outside a buffer of %llu", fn,
                (unsigned long long)offset, (unsigned long long)(offset + n),
                (unsigned long long)buf->len);
  if (n == 0) return AGPU_OK;
  AGPU_CUDA(cudaSetDevice(dev->ordinal));
  float* d = buf->dptr + offset;
  const cudaError_t e =
      to_device ? cudaMemcpyAsync(d, host, n * sizeof(float), cudaMemcpyHostToDevice,
                                  pick_stream(dev, stream))
                : cudaMemcpyAsync(const_cast<void*>(host), d, n * sizeof(float),
                                  cudaMemcpyDeviceToHost, pick_stream(dev, stream));
  return e == cudaSuccess ? AGPU_OK : cuda_status(e, fn);
}

agpu_status agpu_write_async(agpu_device* dev, agpu_buffer* buf, uint64_t offset,
                             const float* host, uint64_t n, void* stream) {
  return copy_async(dev, buf, offset, n, host, true, stream, "agpu_write_async");
}

agpu_status agpu_read_async(agpu_device* dev, const agpu_buffer* buf, uint64_t offset,
                            float* host, uint64_t n, void* stream) {
  return copy_async(dev, buf, offset, n, host, false, stream, "agpu_read_async");
}

agpu_status agpu_selftest_wait_timeout(agpu_device* dev, uint32_t limit_us, void* stream) {
  if (!dev) return fail(AGPU_ERR_INVALID, "agpu_selftest_wait_timeout: NULL device");
  if (limit_us == 0 || limit_us > 1000000u)
    return fail(AGPU_ERR_INVALID, "agpu_selftest_wait_timeout: limit_us %u outside [1, 1000000]",
                limit_us);
  AGPU_CUDA(cudaSetDevice(dev->ordinal));
  wait_timeout_selftest_kernel<<<1, 32, 0, pick_stream(dev, stream)>>>(
      dev->d_status, 1000ull * limit_us, AGPU_SELFTEST_WAIT_CODE);
  return after_launch(dev, "wait_timeout_selftest_kernel");
}

agpu_status agpu_buffer_free(agpu_buffer* buf) {
  if (!buf) return AGPU_OK;
  agpu_device* dev = buf->dev;
  if (dev) {
    cudaSetDevice(dev->ordinal);
    pool_free(dev, buf->dptr, dev->stream);
  }
  delete buf;
  if (dev) device_release(dev);
  return AGPU_OK;
}

uint64_t agpu_buffer_len(const agpu_buffer* buf) { return buf ? buf->len : 0; }

void* agpu_buffer_device_ptr(const agpu_buffer* buf) { return buf ? (void*)buf->dptr : nullptr; }

}  // extern "C"
