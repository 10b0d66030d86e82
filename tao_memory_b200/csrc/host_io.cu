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
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/tao_b200.h"

void tao_set_last_error(const char* msg);

namespace {

__global__ void __launch_bounds__(256) copy16_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src,
                                                     long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dst[i] = src[i];
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

int checked_device(const void* p, const char** why) {
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

extern "C" int tao_copy_host_to_device(void* dst, const void* host_src, size_t bytes, void* stream) {
  int rc = check_args(dst, host_src, bytes);
  if (rc) return rc;
  const char* why = nullptr;
  const void* src = mapped_host(host_src, &why);
  if (!src || !checked_device(dst, &why)) {
    tao_set_last_error(why);
    return TAO_ERR_ARG;
  }
  return launch_copy(dst, src, bytes, stream);
}

extern "C" int tao_copy_device_to_host(void* host_dst, const void* src, size_t bytes, void* stream) {
  int rc = check_args(host_dst, src, bytes);
  if (rc) return rc;
  const char* why = nullptr;
  void* dst = const_cast<void*>(mapped_host(host_dst, &why));
  if (!dst || !checked_device(src, &why)) {
    tao_set_last_error(why);
    return TAO_ERR_ARG;
  }
  return launch_copy(dst, src, bytes, stream);
}
