// Output dequantize fused with the multi-GPU output gather.
//
// The reference dequantizes each graph output after the integer pass
// (quant_container.py:186-193: x = (q - zp) * scale) and, sharded by batch,
// the per-rank shards are then gathered into the full batch.  Here one
// kernel per rank does both: it reads the rank's int32 output rows,
// dequantizes them and stores the float32 rows straight into EVERY rank's
// gather buffer over NVLink peer memory (plain peer stores; no multicast),
// then raises a flag in each peer's buffer.  When a rank's kernel returns,
// the full [world * rows, cols] batch sits in its own buffer.
//
// Buffers: every rank allocates one (qa_peer_buffer_create) and maps every
// other rank's through CUDA IPC (qa_peer_buffer_open).  Layout:
//
//   bytes    0..63   int64 consumed[8]  (written by rank r: it has finished
//                                        copying out its epochs <= value)
//   bytes  128..191  int64 ready[8]     (written by rank r: its rows of the
//                                        epoch = value are in this buffer)
//   bytes  256..259  uint32 arrived     (this rank's CTAs done this launch)
//   bytes 4096..     two data slots of world * rows * cols float32; epoch e
//                    uses slot e & 1
//
// Epochs count from 1.  A launch of epoch e (1) tells every rank that this
// rank consumed epoch e - 1 (the launch starts after every earlier command
// of its stream, among them the copy out of slot (e - 1) & 1), (2) waits
// until every rank has consumed epoch e - 2, the previous user of slot e & 1,
// (3) stores its rows into slot e & 1 of every rank, (4) after its last CTA
// has fenced, publishes ready = e to every rank and (5) waits until every
// rank's ready flag here reaches e.  Waits are bounded by a nanosecond
// budget; a wait that runs out sets the device status word to
// kDeviceTimeout (read by qa_device_status_dev) and the kernel carries on
// without the data of the missing rank.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "qa_common.cuh"

namespace qa {
namespace {

constexpr int kMaxPeers = 8;
constexpr int64_t kPeerHeaderBytes = 4096;
constexpr int kConsumedOffset = 0, kReadyOffset = 128, kArrivedOffset = 256;
constexpr int kGatherThreads = 256;

struct PeerSet {
  char* base[kMaxPeers];
};

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int64_t ld_acquire_sys(const int64_t* p) {
  int64_t v;
  asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(int64_t* p, int64_t v) {
  asm volatile("st.release.sys.global.s64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Waits until flags[r] >= want for r < world; false when the budget ran out.
__device__ bool wait_flags(const int64_t* flags, int world, int64_t want, uint64_t budget_ns) {
  const uint64_t t0 = global_ns();
  for (int r = 0; r < world; ++r) {
    while (ld_acquire_sys(flags + r) < want) {
      if (global_ns() - t0 > budget_ns) return false;
      __nanosleep(256);
    }
  }
  return true;
}

__device__ __forceinline__ float dequant_value(int32_t q, int64_t zp, double scale) {
  return (float)((double)((int64_t)q - zp) * scale);
}

__global__ void __launch_bounds__(kGatherThreads)
    dequant_gather_peers_kernel(const int32_t* __restrict__ q, int64_t q_stride, int64_t zp,
                                double scale, int64_t rows, int64_t cols, PeerSet peers,
                                int world, int rank, int64_t epoch, uint64_t budget_ns,
                                int* status) {
  char* const own = peers.base[rank];
  __shared__ int go;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0)
      for (int r = 0; r < world; ++r)
        st_release_sys(reinterpret_cast<int64_t*>(peers.base[r] + kConsumedOffset) + rank,
                       epoch - 1);
    go = wait_flags(reinterpret_cast<const int64_t*>(own + kConsumedOffset), world, epoch - 2,
                    budget_ns);
    if (!go) atomicExch(status, (int)kDeviceTimeout);
  }
  __syncthreads();
  if (go) {
    const int64_t slot_elems = (int64_t)world * rows * cols;
    const int64_t first = (int64_t)rank * rows * cols + (epoch & 1) * slot_elems;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if ((cols & 3) == 0 && (q_stride & 3) == 0 && (reinterpret_cast<uintptr_t>(q) & 15) == 0) {
      // four columns per thread: one 16-byte load, one 16-byte store per rank
      const int64_t cols4 = cols >> 2;
      for (int64_t i = tid; i < rows * cols4; i += stride) {
        const int64_t r = i / cols4, c = (i - r * cols4) << 2;
        const int4 v = *reinterpret_cast<const int4*>(q + r * q_stride + c);
        const float4 f = make_float4(dequant_value(v.x, zp, scale), dequant_value(v.y, zp, scale),
                                     dequant_value(v.z, zp, scale), dequant_value(v.w, zp, scale));
        const int64_t at = first + r * cols + c;
        for (int p = 0; p < world; ++p)
          *reinterpret_cast<float4*>(reinterpret_cast<float*>(peers.base[p] + kPeerHeaderBytes) +
                                     at) = f;
      }
    } else {
      for (int64_t i = tid; i < rows * cols; i += stride) {
        const int64_t r = i / cols, c = i - r * cols;
        const float f = dequant_value(q[r * q_stride + c], zp, scale);
        for (int p = 0; p < world; ++p)
          reinterpret_cast<float*>(peers.base[p] + kPeerHeaderBytes)[first + r * cols + c] = f;
      }
    }
  }
  // every CTA fences its peer stores before counting itself in; the last
  // one publishes the epoch and waits for the other ranks' rows
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int* arrived = reinterpret_cast<unsigned int*>(own + kArrivedOffset);
    if (atomicAdd(arrived, 1u) == gridDim.x - 1) {
      *arrived = 0;  // the next launch of this stream starts after this one ends
      __threadfence_system();
      for (int r = 0; r < world; ++r)
        st_release_sys(reinterpret_cast<int64_t*>(peers.base[r] + kReadyOffset) + rank, epoch);
      if (!wait_flags(reinterpret_cast<const int64_t*>(own + kReadyOffset), world, epoch,
                      budget_ns))
        atomicExch(status, (int)kDeviceTimeout);
    }
  }
}

}  // namespace
}  // namespace qa

using namespace qa;

QA_API int64_t qa_peer_buffer_header_bytes() { return kPeerHeaderBytes; }

QA_API int qa_peer_buffer_create(int64_t bytes, void** ptr, void* handle) {
  clear_error();
  QA_REQUIRE(ptr && handle, "qa_peer_buffer_create: null output", last_status());
  QA_REQUIRE(bytes >= kPeerHeaderBytes, "qa_peer_buffer_create: smaller than the header",
             last_status());
  if (!thread_context()) return last_status();
  void* p = nullptr;
  QA_CUDA_OR_RETURN(cudaMalloc(&p, (size_t)bytes), last_status());
  if (cuda_failed(cudaMemset(p, 0, (size_t)kPeerHeaderBytes), "cudaMemset")) {
    cudaFree(p);
    return last_status();
  }
  cudaIpcMemHandle_t h;
  if (cuda_failed(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle")) {
    cudaFree(p);
    return last_status();
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return 0;
}

QA_API int qa_peer_buffer_open(const void* handle, void** ptr) {
  clear_error();
  QA_REQUIRE(handle && ptr, "qa_peer_buffer_open: null argument", last_status());
  if (!thread_context()) return last_status();
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  QA_CUDA_OR_RETURN(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), last_status());
  return 0;
}

QA_API int qa_peer_buffer_close(void* ptr) {
  clear_error();
  QA_CUDA_OR_RETURN(cudaIpcCloseMemHandle(ptr), last_status());
  return 0;
}

QA_API int qa_peer_buffer_destroy(void* ptr) {
  clear_error();
  QA_CUDA_OR_RETURN(cudaFree(ptr), last_status());
  return 0;
}

QA_API int qa_dequantize_gather_peers_dev(const void* q, int64_t q_stride, int64_t zp,
                                          double scale, int64_t rows, int64_t cols,
                                          const void* const* bases, int32_t world, int32_t rank,
                                          int64_t epoch, int64_t budget_ns, void* stream) {
  clear_error();
  QA_REQUIRE(q && bases, "qa_dequantize_gather_peers_dev: null pointer", last_status());
  QA_REQUIRE(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world,
             "qa_dequantize_gather_peers_dev: world must lie in [1, 8] and rank below it",
             last_status());
  QA_REQUIRE(rows >= 0 && cols >= 1 && q_stride >= cols,
             "qa_dequantize_gather_peers_dev: bad output shape", last_status());
  QA_REQUIRE(epoch >= 1, "qa_dequantize_gather_peers_dev: epochs count from 1", last_status());
  QA_REQUIRE(budget_ns > 0, "qa_dequantize_gather_peers_dev: budget must be positive",
             last_status());
  PeerSet peers = {};
  for (int r = 0; r < world; ++r) {
    QA_REQUIRE(bases[r] && (reinterpret_cast<uintptr_t>(bases[r]) & 255) == 0,
               "qa_dequantize_gather_peers_dev: every rank's buffer must be mapped and "
               "256-byte aligned",
               last_status());
    peers.base[r] = static_cast<char*>(const_cast<void*>(bases[r]));
  }
  int* status = device_status_word();
  if (!status) return last_status();
  // one launch covers the shard; at least one CTA so the flags always move
  const unsigned grid = grid_for(rows * cols / 4 + 1, kGatherThreads);
  return launch_ex(dequant_gather_peers_kernel, dim3(grid), dim3(kGatherThreads), 0,
                   (cudaStream_t)stream, false, static_cast<const int32_t*>(q), q_stride, zp,
                   scale, rows, cols, peers, (int)world, (int)rank, epoch,
                   (uint64_t)budget_ns, status)
             ? 0
             : last_status();
}
