// Allocation-free variant of the narrow (int16 x int16 -> int32) tensor-core
// GEMM.
//
// Who needs it: callers that must not allocate GPU memory while they run --
// a service that reserves all of its device memory up front and forbids
// allocation afterwards, or a host runtime that hands this library only the
// input and output buffers it manages itself.  The regular entry points grow
// a per-thread device arena and a packing buffer with cudaMalloc on first
// use, which such callers cannot allow.
//
// This entry point packs its operands into a fixed, library-owned scratch
// array instead: a file-scope __device__ array of kNoAllocScratchBytes (16 MiB)
// that every GPU holds from library load until process exit.  Its device
// address is looked up once per device with cudaGetSymbolAddress -- host code
// may not use the array's name as a device address.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "qa_common.cuh"

namespace qa {

size_t umma_gemm_planes_bytes(int64_t M, int64_t N, int64_t K);
bool umma_gemm_i16_i32_into(const int16_t* A, const int16_t* B, int32_t* C, int64_t M,
                            int64_t N, int64_t K, uint8_t* planes, size_t planes_bytes,
                            int32_t* status, cudaStream_t st);

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;

// Byte planes of the packed operands (fully rewritten by every call).
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
// Bounded-wait timeout word of this entry point's kernels (cleared per call).
static __device__ __align__(256) int32_t g_noalloc_status;

constexpr int kMaxDev = 64;
struct DeviceSymbols {
  uint8_t* scratch = nullptr;
  int32_t* status = nullptr;
};
DeviceSymbols g_symbols[kMaxDev];
std::mutex g_symbols_mutex;

// Resolves the device addresses of the static arrays for the current device
// (first call on each device only).
bool device_symbols(DeviceSymbols* out) {
  int dev = 0;
  if (cuda_failed(cudaGetDevice(&dev), "cudaGetDevice")) return false;
  if (dev < 0 || dev >= kMaxDev) {
    set_error(kUnsupported, "device ordinal beyond the no-alloc symbol table");
    return false;
  }
  std::lock_guard<std::mutex> lock(g_symbols_mutex);
  DeviceSymbols& s = g_symbols[dev];
  if (!s.scratch) {
    void* scratch = nullptr;
    void* status = nullptr;
    if (cuda_failed(cudaGetSymbolAddress(&scratch, g_noalloc_scratch),
                    "cudaGetSymbolAddress(scratch)") ||
        cuda_failed(cudaGetSymbolAddress(&status, g_noalloc_status),
                    "cudaGetSymbolAddress(status)"))
      return false;
    s.scratch = static_cast<uint8_t*>(scratch);
    s.status = static_cast<int32_t*>(status);
  }
  *out = s;
  return true;
}

}  // namespace
}  // namespace qa

using namespace qa;

QA_API int64_t qa_noalloc_scratch_bytes(void) { return (int64_t)kNoAllocScratchBytes; }

// Reads and clears this entry point's bounded-wait status word on `stream`
// (a device-to-host copy of one word, then a synchronize of `stream`):
// returns kDeviceTimeout, with the error recorded, when a kernel of an
// earlier call gave up a wait, which leaves that call's C incomplete.
QA_API int qa_noalloc_status_dev(void* stream) {
  clear_error();
  DeviceSymbols sym;
  if (!device_symbols(&sym)) return last_status();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t h = 0;
  if (cuda_failed(cudaMemcpyAsync(&h, sym.status, sizeof(int32_t), cudaMemcpyDeviceToHost, st),
                  "cudaMemcpyAsync(no-alloc status)") ||
      cuda_failed(cudaStreamSynchronize(st), "cudaStreamSynchronize"))
    return last_status();
  if (h != 0) {
    if (cuda_failed(cudaMemsetAsync(sym.status, 0, sizeof(int32_t), st),
                    "cudaMemsetAsync(no-alloc status)") ||
        cuda_failed(cudaStreamSynchronize(st), "cudaStreamSynchronize"))
      return last_status();
    set_error(kDeviceTimeout, "qa_gemm_i16_i32_noalloc_dev: a kernel gave up a bounded wait "
                              "(device status " + std::to_string(h) + "); its output is incomplete");
  }
  return last_status();
}

QA_API int qa_gemm_i16_i32_noalloc_dev(const int16_t* A, const int16_t* B, int32_t* C,
                                       int64_t M, int64_t N, int64_t K, void* stream) {
  clear_error();
  if (M < 0 || N < 0 || K < 0) {
    set_error(kBadArgument, "qa_gemm_i16_i32_noalloc_dev: negative size");
    return last_status();
  }
  if (umma_gemm_planes_bytes(M, N, K) > kNoAllocScratchBytes) {
    set_error(kBadArgument,
              "qa_gemm_i16_i32_noalloc_dev: operands need " +
                  std::to_string(umma_gemm_planes_bytes(M, N, K)) +
                  " bytes of packing scratch; the static maximum is " +
                  std::to_string(kNoAllocScratchBytes));
    return last_status();
  }
  DeviceSymbols sym;
  if (!device_symbols(&sym)) return last_status();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cuda_failed(cudaMemsetAsync(sym.status, 0, sizeof(int32_t), st), "cudaMemsetAsync(status)"))
    return last_status();
  return umma_gemm_i16_i32_into(A, B, C, M, N, K, sym.scratch, kNoAllocScratchBytes, sym.status,
                                st)
             ? 0
             : last_status();
}
