// Small host<->device transfers of a decode step done by the SMs over the host link.
//
// One decode step of a serving batch moves tens of kilobytes each way (q, k, v, raw_q,
// raw_k in; the fused output back).  At that size a copy-engine transfer is latency-
// bound (measured on B200: about 23 us for 61 KB in, 9 us for 12 KB out, next to a
// 22 us step).  Page-locked host memory that CUDA has mapped into the device's
// address space can instead be read and written by a kernel directly: every thread
// moves 16 bytes, all loads are in flight at once, so the transfer costs about one
// round trip over the link plus a launch.
//
// The host pointer is checked with cudaPointerGetAttributes before any launch: it must
// be page-locked host memory with a device mapping, 16-byte aligned, and the size a
// multiple of 16 bytes; anything else returns TAO_ERR_ARG and nothing is accessed.
// The device side must be one allocation holding all `bytes` (its extent is asked of
// the driver, cuMemGetAddressRange); the caller keeps the host range in bounds.
#include <cuda.h>
#include <cuda_runtime.h>

#include <immintrin.h>

#include <chrono>
#include <cstdint>
#include <mutex>

#include "../../include/tao_b200.h"

void tao_set_last_error(const char* msg);

namespace {

__global__ void __launch_bounds__(256) copy16_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src,
                                                     long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

// Up to kMaxCopies buffers in one launch (a decode step's five operands).
constexpr int kMaxCopies = 8;
struct CopyList {
  uint4* dst[kMaxCopies];
  const uint4* src[kMaxCopies];
  long long n[kMaxCopies];  // 16-byte vectors
  int count;
};

__global__ void __launch_bounds__(256) copy16_many_kernel(CopyList L) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long first = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  for (int c = 0; c < L.count; ++c) {
    uint4* __restrict__ d = L.dst[c];
    const uint4* __restrict__ sp = L.src[c];
    for (long long i = first; i < L.n[c]; i += stride) d[i] = sp[i];
  }
}

// Device address of mapped page-locked host memory, or nullptr.
const void* mapped_host(const void* host, const char** why) {
  cudaPointerAttributes attr{};
  if (cudaPointerGetAttributes(&attr, host) != cudaSuccess) {
    cudaGetLastError();
    *why = "host buffer is not known to CUDA (not page-locked)";
    return nullptr;
  }
  if (attr.type != cudaMemoryTypeHost) {
    *why = "host buffer must be page-locked host memory";
    return nullptr;
  }
  if (attr.devicePointer == nullptr) {
    *why = "page-locked host buffer has no device mapping";
    return nullptr;
  }
  return attr.devicePointer;
}

using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q{};
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(p);
  });
  return fn;
}

int checked_device(const void* p, size_t bytes, const char** why) {
  cudaPointerAttributes attr{};
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    cudaGetLastError();
    *why = "device buffer is not known to CUDA";
    return 0;
  }
  if (attr.type != cudaMemoryTypeDevice) {
    *why = "device buffer must be device memory";
    return 0;
  }
  int current = -1;
  if (cudaGetDevice(&current) != cudaSuccess || attr.device != current) {
    cudaGetLastError();
    *why = "device buffer is not on the calling thread's current device";
    return 0;
  }
  AddressRangeFn range = address_range_fn();
  CUdeviceptr base = 0;
  size_t size = 0;
  if (!range || range(&base, &size, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS) {
    *why = "device buffer extent is unknown to the driver";
    return 0;
  }
  const uintptr_t first = reinterpret_cast<uintptr_t>(p);
  if (first < base || bytes > size || first - base > size - bytes) {
    *why = "transfer runs past the end of the device allocation";
    return 0;
  }
  return 1;
}

int launch_copy(void* dst, const void* src, size_t bytes, void* stream) {
  const long long n = (long long)(bytes / 16);
  if (n == 0) return TAO_OK;
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  copy16_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(dst), static_cast<const uint4*>(src), n);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    tao_set_last_error(cudaGetErrorString(e));
    return TAO_ERR_CUDA;
  }
  return TAO_OK;
}

int check_args(const void* a, const void* b, size_t bytes) {
  if (!a || !b) {
    tao_set_last_error("null buffer");
    return TAO_ERR_ARG;
  }
  if (((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15) || (bytes & 15)) {
    tao_set_last_error("host transfer buffers must be 16-byte aligned and a multiple of 16 bytes");
    return TAO_ERR_ARG;
  }
  return TAO_OK;
}

}  // namespace

extern "C" int tao_host_device_pointer(const void* host, void** device) {
  if (!host || !device) {
    tao_set_last_error("null host buffer or result pointer");
    return TAO_ERR_ARG;
  }
  const char* why = nullptr;
  const void* p = mapped_host(host, &why);
  if (!p) {
    tao_set_last_error(why);
    return TAO_ERR_ARG;
  }
  *device = const_cast<void*>(p);
  return TAO_OK;
}

extern "C" int tao_host_wait(const void* word, int value, long long timeout_us) {
  if (!word) {
    tao_set_last_error("null completion word");
    return TAO_ERR_ARG;
  }
  const volatile int* p = static_cast<const volatile int*>(word);
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    for (int i = 0; i < 64; ++i) {
      if ((int)((unsigned)*p - (unsigned)value) >= 0) return TAO_OK;
      _mm_pause();
    }
    if (std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0).count() >
        timeout_us) {
      tao_set_last_error("host wait for a completion word expired");
      return TAO_ERR_TIMEOUT;
    }
  }
}

extern "C" int tao_graph_launch(void* graph_exec, void* stream) {
  if (!graph_exec) {
    tao_set_last_error("null graph");
    return TAO_ERR_ARG;
  }
  cudaError_t e = cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph_exec), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    cudaGetLastError();
    tao_set_last_error(cudaGetErrorString(e));
    return TAO_ERR_CUDA;
  }
  return TAO_OK;
}

extern "C" int tao_copy_host_to_device(void* dst, const void* host_src, size_t bytes, void* stream) {
  int rc = check_args(dst, host_src, bytes);
  if (rc) return rc;
  const char* why = nullptr;
  const void* src = mapped_host(host_src, &why);
  if (!src || !checked_device(dst, bytes, &why)) {
    tao_set_last_error(why);
    return TAO_ERR_ARG;
  }
  return launch_copy(dst, src, bytes, stream);
}

extern "C" int tao_copy_host_to_device_many(void* const* dst, const void* const* host_src, const size_t* bytes,
                                            int n, void* stream) {
  if (!dst || !host_src || !bytes || n <= 0 || n > kMaxCopies) {
    tao_set_last_error("host copy list: null arrays or count outside 1..8");
    return TAO_ERR_ARG;
  }
  CopyList L{};
  long long most = 0;
  for (int c = 0; c < n; ++c) {
    int rc = check_args(dst[c], host_src[c], bytes[c]);
    if (rc) return rc;
    const char* why = nullptr;
    const void* src = mapped_host(host_src[c], &why);
    if (!src || !checked_device(dst[c], bytes[c], &why)) {
      tao_set_last_error(why);
      return TAO_ERR_ARG;
    }
    L.dst[c] = static_cast<uint4*>(dst[c]);
    L.src[c] = static_cast<const uint4*>(src);
    L.n[c] = (long long)(bytes[c] / 16);
    if (L.n[c] > most) most = L.n[c];
  }
  L.count = n;
  if (most == 0) return TAO_OK;
  long long blocks = (most + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  copy16_many_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(L);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    tao_set_last_error(cudaGetErrorString(e));
    return TAO_ERR_CUDA;
  }
  return TAO_OK;
}

extern "C" int tao_copy_device_to_host(void* host_dst, const void* src, size_t bytes, void* stream) {
  int rc = check_args(host_dst, src, bytes);
  if (rc) return rc;
  const char* why = nullptr;
  void* dst = const_cast<void*>(mapped_host(host_dst, &why));
  if (!dst || !checked_device(src, bytes, &why)) {
    tao_set_last_error(why);
    return TAO_ERR_ARG;
  }
  return launch_copy(dst, src, bytes, stream);
}
