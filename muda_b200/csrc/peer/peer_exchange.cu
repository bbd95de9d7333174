// peer_exchange.cu — x all-gather of the distributed SpMV over NVLink peer memory.
//
// Each rank's exchange buffer (header + two x buffers) is mapped into every other
// rank's address space with CUDA IPC.  One kernel per epoch and rank:
//   1. own block: every CTA copies its share of x_local into the rank's epoch buffer
//      and counts itself done in header word kArriveWord; the CTA that completes the
//      count (no CTA waits for another) resets it and announces: st.release.sys of
//      the epoch into word `rank` of every peer's header;
//   2. pull: CTAs take (peer, 32 KB chunk) items; thread 0 waits for the peer's
//      announcement with ld.acquire.sys (bounded by %globaltimer, about one second),
//      then the CTA copies the chunk from the peer's buffer with 16-byte loads over
//      NVLink into the same offsets of this rank's buffer.
// No kernel waits on another kernel of the same GPU: the flags are written by the
// other ranks' kernels, each on its own GPU.  A wait that runs out records the peer
// in the status word and skips its chunk, so the kernel always ends.
#pragma GCC visibility push(default)
#include "mb200_peer.h"
#pragma GCC visibility pop

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "common/device.hpp"

namespace {

constexpr std::size_t kHeaderBytes = 256;
constexpr int kThreads = 256;
constexpr int kVecPerThread = 8;
constexpr int kArriveWord = MB200_PEER_STATUS_WORD + 1;  // CTAs done with the own block
constexpr std::size_t kChunkFloats = static_cast<std::size_t>(kThreads) * kVecPerThread * 4;
constexpr unsigned long long kWaitNs = 1000000000ull;  // about one second per peer

static_assert(MB200_PEER_STATUS_WORD >= MB200_PEER_MAX_RANKS &&
                  (kArriveWord + 1) * 4 <= static_cast<int>(kHeaderBytes),
              "header layout");
static_assert(sizeof(cudaIpcMemHandle_t) == MB200_PEER_HANDLE_BYTES, "IPC handle size");

struct PullArgs {
  void* bases[MB200_PEER_MAX_RANKS];
  const float* x_local;
  int world, rank;
  unsigned epoch;
  unsigned long long count, block;
};

__device__ __forceinline__ unsigned* header(void* base) { return static_cast<unsigned*>(base); }

__device__ __forceinline__ float* buffer(void* base, unsigned long long count, unsigned epoch) {
  return reinterpret_cast<float*>(static_cast<char*>(base) + kHeaderBytes) +
         (epoch & 1u) * count;
}

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned load_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void store_release(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// True once peer `p` has announced `epoch` (epochs compared modulo 2^32).  A peer
// whose status bit is set (a wait for it ran out since the status was last taken)
// is skipped at once.
__device__ bool wait_announced(unsigned* own_header, int p, unsigned epoch) {
  const unsigned* f = own_header + p;
  if (static_cast<int>(load_acquire(f) - epoch) >= 0) return true;
  volatile unsigned* st = own_header + MB200_PEER_STATUS_WORD;
  if ((*st >> p) & 1u) return false;
  const unsigned long long t0 = now_ns();
  for (;;) {
    __nanosleep(256);
    if (static_cast<int>(load_acquire(f) - epoch) >= 0) return true;
    if (now_ns() - t0 > kWaitNs) {
      atomicOr(own_header + MB200_PEER_STATUS_WORD, 1u << p);
      return false;
    }
  }
}

// dst[i] = src[i] for i in [lo, hi) by this CTA (16-byte copies when VEC).
template <bool VEC>
__device__ __forceinline__ void copy_range(const float* src, float* dst, unsigned long long lo,
                                           unsigned long long hi) {
  if constexpr (VEC) {
    const float4* s4 = reinterpret_cast<const float4*>(src + lo);
    float4* d4 = reinterpret_cast<float4*>(dst + lo);
    const long long n4 = static_cast<long long>((hi - lo) / 4);
    for (long long i0 = 0; i0 < n4; i0 += static_cast<long long>(kThreads) * kVecPerThread) {
      float4 v[kVecPerThread];
#pragma unroll
      for (int u = 0; u < kVecPerThread; ++u) {
        const long long i = i0 + threadIdx.x + static_cast<long long>(u) * kThreads;
        if (i < n4) v[u] = s4[i];
      }
#pragma unroll
      for (int u = 0; u < kVecPerThread; ++u) {
        const long long i = i0 + threadIdx.x + static_cast<long long>(u) * kThreads;
        if (i < n4) d4[i] = v[u];
      }
    }
  } else {
    for (unsigned long long i = lo + threadIdx.x; i < hi; i += kThreads) dst[i] = src[i];
  }
}

template <bool VEC>
__global__ void __launch_bounds__(kThreads) peer_pull(const PullArgs a) {
  __shared__ int ready;
  unsigned* own = header(a.bases[a.rank]);
  float* dst_buf = buffer(a.bases[a.rank], a.count, a.epoch);
  // 1. this CTA's share of the own block (a multiple of 4 floats when VEC)
  {
    const unsigned long long per =
        ((a.block + gridDim.x - 1) / gridDim.x + 3) / 4 * 4;
    const unsigned long long lo = blockIdx.x * per < a.block ? blockIdx.x * per : a.block;
    const unsigned long long hi = lo + per < a.block ? lo + per : a.block;
    const unsigned long long off = static_cast<unsigned long long>(a.rank) * a.block;
    copy_range<VEC>(a.x_local, dst_buf + off, lo, hi);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) ready = atomicAdd(own + kArriveWord, 1u) == gridDim.x - 1 ? 1 : 0;
    __syncthreads();
    if (ready) {  // the last CTA: the whole own block is in place
      if (threadIdx.x == 0) own[kArriveWord] = 0;
      if (static_cast<int>(threadIdx.x) < a.world && static_cast<int>(threadIdx.x) != a.rank) {
        __threadfence_system();
        store_release(header(a.bases[threadIdx.x]) + a.rank, a.epoch);
      }
    }
    __syncthreads();
  }
  // 2. the peers' blocks
  const unsigned long long chunks = (a.block + kChunkFloats - 1) / kChunkFloats;
  const unsigned long long items = static_cast<unsigned long long>(a.world - 1) * chunks;
  for (unsigned long long it = blockIdx.x; it < items; it += gridDim.x) {
    const int q = static_cast<int>(it / chunks);
    const int peer = q < a.rank ? q : q + 1;
    const unsigned long long c = it % chunks;
    if (threadIdx.x == 0) ready = wait_announced(own, peer, a.epoch) ? 1 : 0;
    __syncthreads();
    if (ready) {
      const unsigned long long lo = static_cast<unsigned long long>(peer) * a.block +
                                    c * kChunkFloats;
      const unsigned long long end = static_cast<unsigned long long>(peer) * a.block + a.block;
      const unsigned long long hi = lo + kChunkFloats < end ? lo + kChunkFloats : end;
      // lo and hi are multiples of 4 when VEC (block % 4 == 0)
      copy_range<VEC>(buffer(a.bases[peer], a.count, a.epoch), dst_buf, lo, hi);
    }
    __syncthreads();
  }
}

mb200PeerStatus_t cuda_status(cudaError_t e) {
  return e == cudaSuccess ? MB200_PEER_SUCCESS : MB200_PEER_CUDA_ERROR;
}

}  // namespace

extern "C" {

mb200PeerStatus_t mb200PeerAlloc(size_t count, void** base, void* handle) {
  if (base == nullptr || handle == nullptr || count == 0 ||
      count > (std::size_t{1} << 40) / 8)
    return MB200_PEER_INVALID_VALUE;
  *base = nullptr;
  const std::size_t bytes = kHeaderBytes + 2 * count * sizeof(float);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return MB200_PEER_CUDA_ERROR;
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    (void)cudaFree(p);
    return MB200_PEER_CUDA_ERROR;
  }
  std::memcpy(handle, &h, sizeof(h));
  *base = p;
  return MB200_PEER_SUCCESS;
}

mb200PeerStatus_t mb200PeerOpen(const void* handle, void** peer_base) {
  if (handle == nullptr || peer_base == nullptr) return MB200_PEER_INVALID_VALUE;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *peer_base = nullptr;
  return cuda_status(cudaIpcOpenMemHandle(peer_base, h, cudaIpcMemLazyEnablePeerAccess));
}

mb200PeerStatus_t mb200PeerClose(void* peer_base) {
  if (peer_base == nullptr) return MB200_PEER_INVALID_VALUE;
  return cuda_status(cudaIpcCloseMemHandle(peer_base));
}

mb200PeerStatus_t mb200PeerFree(void* base) {
  if (base == nullptr) return MB200_PEER_INVALID_VALUE;
  return cuda_status(cudaFree(base));
}

float* mb200PeerBuffer(void* base, size_t count, unsigned epoch) {
  if (base == nullptr) return nullptr;
  return reinterpret_cast<float*>(static_cast<char*>(base) + kHeaderBytes) + (epoch & 1u) * count;
}

mb200PeerStatus_t mb200PeerAllgather(void* const* bases, int world, int rank, size_t count,
                                     size_t block, unsigned epoch, const float* x_local,
                                     cudaStream_t stream) {
  if (bases == nullptr || world < 1 || world > MB200_PEER_MAX_RANKS || rank < 0 ||
      rank >= world || block == 0 || epoch == 0 || x_local == nullptr ||
      static_cast<unsigned long long>(world) * block > count)
    return MB200_PEER_INVALID_VALUE;
  PullArgs a{};
  for (int p = 0; p < world; ++p) {
    if (bases[p] == nullptr) return MB200_PEER_INVALID_VALUE;
    a.bases[p] = bases[p];
  }
  a.x_local = x_local;
  a.world = world;
  a.rank = rank;
  a.epoch = epoch;
  a.count = count;
  a.block = block;
  const int sms = mb200::sm_count(mb200::current_device());
  const unsigned grid = static_cast<unsigned>((sms > 0 ? sms : 148) * 2);
  const bool vec = block % 4 == 0 && count % 4 == 0 &&
                   reinterpret_cast<std::uintptr_t>(x_local) % 16 == 0;
  if (vec)
    peer_pull<true><<<grid, kThreads, 0, stream>>>(a);
  else
    peer_pull<false><<<grid, kThreads, 0, stream>>>(a);
  return cuda_status(cudaGetLastError());
}

mb200PeerStatus_t mb200PeerTakeStatus(void* base, unsigned* status) {
  if (base == nullptr || status == nullptr) return MB200_PEER_INVALID_VALUE;
  unsigned* word = static_cast<unsigned*>(base) + MB200_PEER_STATUS_WORD;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(status, word, sizeof(unsigned), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemset(word, 0, sizeof(unsigned));
  return cuda_status(e);
}

}  // extern "C"
