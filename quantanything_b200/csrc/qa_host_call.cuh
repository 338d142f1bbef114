// HostCall: staging of one host-pointer ABI call.
//
// The reference ABI passes host buffers and expects the outputs on return.
// A HostCall lays every input and output out in the calling thread's device
// arena (256-byte aligned slots), copies inputs host->device on the thread's
// stream, and after the caller enqueues its kernels copies outputs back and
// synchronizes.  Steady-state calls allocate nothing.
//
// Usage:
//   HostCall hc;
//   auto a = hc.input(host_a, n);      // slot handles, no device memory yet
//   auto o = hc.output(host_out, n);
//   if (!hc.upload()) return;          // arena sized, inputs copied
//   kernel<<<..., hc.stream()>>>(hc.dev(a), hc.dev(o), n);
//   hc.download();                     // outputs copied back, stream synced
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "qa_common.cuh"

namespace qa {

template <typename T>
struct Slot {
  size_t index;
};

class HostCall {
 public:
  HostCall() : ctx_(thread_context()) {}

  template <typename T>
  Slot<T> input(const T* host, int64_t count) {
    return Slot<T>{add(host, nullptr, (size_t)count * sizeof(T))};
  }
  template <typename T>
  Slot<T> output(T* host, int64_t count) {
    return Slot<T>{add(nullptr, host, (size_t)count * sizeof(T))};
  }
  template <typename T>
  Slot<T> scratch(int64_t count) {
    return Slot<T>{add(nullptr, nullptr, (size_t)count * sizeof(T))};
  }

  bool upload() {
    if (!ctx_) return false;
    if (!arena_reserve(ctx_, offset_)) return false;
    base_ = static_cast<char*>(ctx_->arena);
    for (auto& s : slots_) {
      if (s.host_in && s.bytes &&
          cuda_failed(cudaMemcpyAsync(base_ + s.offset, s.host_in, s.bytes,
                                      cudaMemcpyHostToDevice, ctx_->stream),
                      "cudaMemcpyAsync(H2D)"))
        return false;
    }
    return true;
  }

  template <typename T>
  T* dev(Slot<T> s) const {
    return reinterpret_cast<T*>(base_ + slots_[s.index].offset);
  }

  bool download() {
    for (auto& s : slots_) {
      if (s.host_out && s.bytes &&
          cuda_failed(cudaMemcpyAsync(s.host_out, base_ + s.offset, s.bytes,
                                      cudaMemcpyDeviceToHost, ctx_->stream),
                      "cudaMemcpyAsync(D2H)"))
        return false;
    }
    if (cuda_failed(cudaStreamSynchronize(ctx_->stream), "cudaStreamSynchronize")) return false;
    return check_device_status(ctx_->stream);
  }

  cudaStream_t stream() const { return ctx_ ? ctx_->stream : nullptr; }

 private:
  struct Entry {
    const void* host_in;
    void* host_out;
    size_t offset;
    size_t bytes;
  };

  size_t add(const void* in, void* out, size_t bytes) {
    slots_.push_back(Entry{in, out, offset_, bytes});
    offset_ += align256(bytes ? bytes : 1);
    return slots_.size() - 1;
  }

  ThreadContext* ctx_;
  std::vector<Entry> slots_;
  size_t offset_ = 0;
  char* base_ = nullptr;
};

}  // namespace qa
