// Shared host-side plumbing of the kernel library: the per-thread status
// word behind qa_last_status()/qa_last_error(), device selection, a per
// thread CUDA stream and grow-only device scratch arena for the host-pointer
// entry points, and launch helpers.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>

#define QA_API extern "C" __attribute__((visibility("default")))

namespace qa {

// ------------------------------------------------------------- status --
enum Status : int {
  kOk = 0,
  kCudaError = 1,
  kBadArgument = 2,
  kDeviceTimeout = 3,
  kUnsupported = 4,
};

void set_error(int status, const std::string& msg);  // aborts in abort mode
void clear_error();
int last_status();

// Returns true (and records the error) when `e` is not cudaSuccess.
bool cuda_failed(cudaError_t e, const char* what);

#define QA_CUDA_OR_RETURN(expr, ...)                       \
  do {                                                     \
    if (::qa::cuda_failed((expr), #expr)) return __VA_ARGS__; \
  } while (0)

#define QA_REQUIRE(cond, msg, ...)                         \
  do {                                                     \
    if (!(cond)) {                                         \
      ::qa::set_error(::qa::kBadArgument, (msg));          \
      return __VA_ARGS__;                                  \
    }                                                      \
  } while (0)

// ------------------------------------------------------- thread context --
// Everything a host-pointer entry point needs on the calling thread: the
// selected device, a private non-blocking stream and a scratch arena that
// only grows (so steady-state calls allocate nothing).
struct ThreadContext {
  int device = -1;
  cudaStream_t stream = nullptr;
  void* arena = nullptr;
  size_t arena_bytes = 0;
  int* dev_status = nullptr;  // device-side error word (timeouts)
};

// Binds the calling thread to its device and returns its context, or
// nullptr (with the error recorded) if no device is usable.
ThreadContext* thread_context();

// Carves `bytes` (rounded to 256) out of the arena; `offset` accumulates.
// Returns false (error recorded) if the arena cannot grow.
bool arena_reserve(ThreadContext* ctx, size_t total_bytes);

inline size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

// Number of SMs of the current device (cached).
int sm_count();

// Device pointer of a per-device int32 error word that kernels set when a
// bounded wait gives up (kDeviceTimeout) instead of trapping.
int* device_status_word();
// Reads and clears the device error word after a synchronize; records an
// error and returns false if a kernel reported one.
bool check_device_status(cudaStream_t stream);

// Launches `kern` on `st`; with `pdl` the launch may overlap the previous
// kernel of the stream (programmatic dependent launch): the kernel must call
// griddepcontrol.wait before reading anything that kernel wrote.
template <typename... KArgs, typename... Args>
bool launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
               bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return !cuda_failed(cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...),
                      "cudaLaunchKernelEx");
}

inline unsigned grid_for(int64_t n, int threads, int per_thread = 1) {
  int64_t blocks = (n + (int64_t)threads * per_thread - 1) / ((int64_t)threads * per_thread);
  int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (unsigned)blocks;
}

}  // namespace qa
