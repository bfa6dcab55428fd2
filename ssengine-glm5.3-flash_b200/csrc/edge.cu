// Stage edge over NVLink: the sender's kernels store activation rows straight into the receiver's ring slot (a CUDA
// IPC mapping of the peer's memory), and 32-bit flag words order it.
//
// Reference behaviour (ssengine/runtime/transport.py:205-335 `CePipe`): the sender copies a finished microbatch into
// slot (n-1) % K of the receiver's ring by copy engine, then writes ready[slot] = n; the receiver's stream waits
// ready[slot] >= n before its forward and writes free[slot] = n back after; the sender waits free[slot] >= n - K before
// reusing the slot; stage 0 waits exits >= n - depth (the in-flight gate) written by the last stage. Here the waits are
// one-thread kernels with a time limit (the status word receives 4 and the kernel returns instead of hanging), the
// writes are release stores at system scope, and the copy is an SM kernel of 16-byte stores into peer memory (or the
// producing kernel writes the peer slot itself). No cluster multicast, no NCCL.
#include <cstring>

#include "../../include/ssengine_b200.h"
#include "common.cuh"
#include "ops.h"

namespace ssb {
namespace {

SSB_DEVICE uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
SSB_DEVICE void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits until (int32)(*flag - value) >= 0, at most timeout_ns of %globaltimer; on expiry raises kErrTimeout.
__global__ void flag_wait_kernel(const uint32_t* flag, uint32_t value, unsigned long long timeout_ns, int32_t* status) {
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (static_cast<int32_t>(ld_acquire_sys(flag) - value) >= 0) return;
    if (globaltimer() - t0 > timeout_ns) {
      raise_status(status, kErrTimeout);
      return;
    }
    __nanosleep(256);
  }
}

// Everything the stream did before (earlier kernels' stores, local or peer) is visible before the flag.
__global__ void flag_write_kernel(uint32_t* flag, uint32_t value) {
  __threadfence_system();
  st_release_sys(flag, value);
}

// dst, src 16-byte aligned; bytes % 16 == 0; grid-stride 16-byte copies (dst may be a peer mapping).
__global__ void p2p_copy_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src, int64_t n16) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = __ldg(src + i);
}

}  // namespace
}  // namespace ssb

using ssb::kErrArgs;
using ssb::kErrCuda;
using ssb::kOk;

extern "C" {

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

int ssb_ipc_export(const void* dev_ptr, uint8_t* handle64, int64_t* offset) {
  if (dev_ptr == nullptr || handle64 == nullptr || offset == nullptr) return kErrArgs;
  static AddressRangeFn range = nullptr;
  if (range == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return ssb::kErrNoDriver;
    range = reinterpret_cast<AddressRangeFn>(p);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return kErrCuda;
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return kErrCuda;
  static_assert(sizeof(h) == 64, "IPC handle size");
  memcpy(handle64, &h, 64);
  return kOk;
}

int ssb_ipc_open(const uint8_t* handle64, void** dev_ptr) {
  if (handle64 == nullptr || dev_ptr == nullptr) return kErrArgs;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, 64);
  if (cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return kErrCuda;
  return kOk;
}

int ssb_ipc_close(void* dev_ptr) {
  if (dev_ptr == nullptr) return kErrArgs;
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? kOk : kErrCuda;
}

int ssb_flag_wait(const uint32_t* flag, uint32_t value, int64_t timeout_ns, int32_t* status, void* stream) {
  if (flag == nullptr || timeout_ns <= 0) return kErrArgs;
  ssb::flag_wait_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(flag, value,
                                                                        static_cast<unsigned long long>(timeout_ns), status);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int ssb_flag_write(uint32_t* flag, uint32_t value, void* stream) {
  if (flag == nullptr) return kErrArgs;
  ssb::flag_write_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(flag, value);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int ssb_p2p_copy(void* dst, const void* src, int64_t bytes, void* stream) {
  if (dst == nullptr || src == nullptr || bytes < 0 || (bytes & 15) || (reinterpret_cast<uintptr_t>(dst) & 15) ||
      (reinterpret_cast<uintptr_t>(src) & 15))
    return kErrArgs;
  if (bytes == 0) return kOk;
  const int64_t n16 = bytes / 16;
  const int sms = ssb::device_sm_count();
  const int64_t want = (n16 + 255) / 256;
  const int grid = static_cast<int>(want < 4LL * sms ? want : 4LL * sms);
  ssb::p2p_copy_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint4*>(dst),
                                                                           static_cast<const uint4*>(src), n16);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // extern "C"
