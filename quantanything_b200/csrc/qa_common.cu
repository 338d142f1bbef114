// Status channel, device selection and per-thread resources.
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "qa_common.cuh"

namespace qa {

namespace {

thread_local int t_status = kOk;
thread_local std::string t_message;
int g_abort_on_error = -1;  // -1: not yet read from the environment
std::mutex g_mutex;

bool abort_mode() {
  if (g_abort_on_error < 0) {
    const char* v = std::getenv("QA_ON_ERROR");
    g_abort_on_error = (v && std::strcmp(v, "record") == 0) ? 0 : 1;
  }
  return g_abort_on_error == 1;
}

// The device host-pointer calls run on when the thread never called
// qa_set_device: $QA_DEVICE if set, else the calling thread's current CUDA
// device (so a caller that selected its GPU is never switched away from it).
int default_device() {
  const char* v = std::getenv("QA_DEVICE");
  if (v) return std::atoi(v);
  int cur = 0;
  if (cudaGetDevice(&cur) != cudaSuccess) return 0;
  return cur;
}

thread_local ThreadContext t_ctx;
thread_local int t_requested_device = -1;

constexpr int kMaxDevices = 64;
int* g_status_words[kMaxDevices] = {nullptr};
int g_sm_count[kMaxDevices] = {0};

}  // namespace

void set_error(int status, const std::string& msg) {
  t_status = status;
  t_message = msg;
  if (abort_mode()) {
    std::fprintf(stderr, "libqa_kernels: fatal: %s\n", msg.c_str());
    std::fflush(stderr);
    std::abort();
  }
}

void clear_error() {
  t_status = kOk;
  t_message.clear();
}

int last_status() { return t_status; }

bool cuda_failed(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return false;
  set_error(kCudaError, std::string(what) + ": " + cudaGetErrorString(e));
  return true;
}

ThreadContext* thread_context() {
  ThreadContext* ctx = &t_ctx;
  const int want = t_requested_device >= 0 ? t_requested_device : default_device();
  if (ctx->device != want) {
    int count = 0;
    if (cuda_failed(cudaGetDeviceCount(&count), "cudaGetDeviceCount")) return nullptr;
    if (want < 0 || want >= count || want >= kMaxDevices) {
      set_error(kBadArgument, "QA device ordinal " + std::to_string(want) +
                                  " out of range (" + std::to_string(count) + " visible)");
      return nullptr;
    }
    if (cuda_failed(cudaSetDevice(want), "cudaSetDevice")) return nullptr;
    // A thread that switches devices drops its old stream/arena.
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    if (ctx->arena) cudaFree(ctx->arena);
    ctx->stream = nullptr;
    ctx->arena = nullptr;
    ctx->arena_bytes = 0;
    if (cuda_failed(cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking),
                    "cudaStreamCreate"))
      return nullptr;
    ctx->device = want;
  } else {
    if (cuda_failed(cudaSetDevice(want), "cudaSetDevice")) return nullptr;
  }
  return ctx;
}

bool arena_reserve(ThreadContext* ctx, size_t total_bytes) {
  if (total_bytes <= ctx->arena_bytes) return true;
  size_t want = ctx->arena_bytes ? ctx->arena_bytes : (size_t(64) << 20);
  while (want < total_bytes) want *= 2;
  if (ctx->arena) {
    if (cuda_failed(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize")) return false;
    cudaFree(ctx->arena);
    ctx->arena = nullptr;
    ctx->arena_bytes = 0;
  }
  if (cuda_failed(cudaMalloc(&ctx->arena, want), "cudaMalloc(arena)")) return false;
  ctx->arena_bytes = want;
  return true;
}

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sm_count[dev] = n > 0 ? n : 148;
  }
  return g_sm_count[dev];
}

int* device_status_word() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_status_words[dev]) {
    int* p = nullptr;
    if (cuda_failed(cudaMalloc(&p, sizeof(int)), "cudaMalloc(status)")) return nullptr;
    cudaMemset(p, 0, sizeof(int));
    cudaDeviceSynchronize();
    g_status_words[dev] = p;
  }
  return g_status_words[dev];
}

bool check_device_status(cudaStream_t stream) {
  int* word = device_status_word();
  if (!word) return false;
  int h = 0;
  if (cuda_failed(cudaMemcpyAsync(&h, word, sizeof(int), cudaMemcpyDeviceToHost, stream),
                  "cudaMemcpyAsync(status)"))
    return false;
  if (cuda_failed(cudaStreamSynchronize(stream), "cudaStreamSynchronize")) return false;
  if (h != 0) {
    cudaMemsetAsync(word, 0, sizeof(int), stream);
    cudaStreamSynchronize(stream);
    set_error(kDeviceTimeout,
              "a kernel gave up a bounded wait (device status " + std::to_string(h) + ")");
    return false;
  }
  return true;
}

}  // namespace qa

// ------------------------------------------------------------- C API --
QA_API int qa_last_status(void) { return qa::last_status(); }

QA_API const char* qa_last_error(void) {
  return qa::last_status() == qa::kOk ? "" : qa::t_message.c_str();
}

QA_API void qa_clear_error(void) { qa::clear_error(); }

QA_API void qa_set_error_mode(int abort_on_error) {
  qa::g_abort_on_error = abort_on_error ? 1 : 0;
}

QA_API int qa_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

QA_API int qa_set_device(int ordinal) {
  qa::t_requested_device = ordinal;
  return qa::thread_context() ? 0 : qa::last_status();
}

QA_API int qa_get_device(void) {
  return qa::t_requested_device >= 0 ? qa::t_requested_device : qa::default_device();
}

// Reference threading introspection (qa_kernels.cpp:233-249).
QA_API int qa_num_threads(void) {
  const int n = qa_device_count();
  return n > 0 ? n : 1;
}
QA_API void qa_set_num_threads(int n) { (void)n; }
QA_API int qa_has_openmp(void) { return 0; }
