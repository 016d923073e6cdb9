// Peer-memory reduce-scatter of the parameter-block-sharded forward (one process per GPU, NVLink /
// NVSwitch peer access).
//
// Each rank's down projection stores the partial output rows of token slice o straight into rank o's
// receive buffer (slot = the writing rank), over NVLink, as its epilogue produces them: the transfer
// overlaps the contraction tile by tile instead of following it as a separate collective.  A one-warp
// kernel then raises the writer's flag on every rank (release, system scope), and each rank's combine
// kernel waits (bounded) for all flags and sums the world slots of its own rows in rank order.
//
// Receive buffer of one rank (one cudaMalloc, shared through CUDA IPC):
//   [0, kPeerFlagBytes)      flags[w] = epoch of the last call whose partial rank w finished writing here
//   then 2 parities x world slots x rows x D partials (bf16 or fp32)
// Calls alternate parities, so a writer of call e+1 never touches the slots that the combine of call e
// reads: a rank starts call e+1 only after its own combine of call e, which waited for every rank's
// flag of call e, which each rank raised after its combine of call e-1 (same-stream order) -- so when
// call e+1 writes parity (e+1)%2 = (e-1)%2, the combine of call e-1 on every rank has finished.  Flags
// hold monotonically increasing epochs (a wait accepts flag >= epoch), so no reset is needed.
#include "fp_internal.cuh"

#include <algorithm>
#include <cstring>

namespace fp {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Thread w raises this rank's flag on rank w (after every store of the preceding kernels of the stream).
__global__ void peer_signal_kernel(PeerFlags f, uint32_t epoch) {
  const int w = threadIdx.x;
  __threadfence_system();
  if (w < f.world && f.flag[w]) st_release_sys(f.flag[w], epoch);
}

// Sum of the world slots of this rank's rows in rank order; every CTA first waits (bounded) until all
// ranks' flags reached `epoch`.  8 elements per thread and step.
template <bool kInF32, bool kOutF32>
__global__ void __launch_bounds__(256) peer_combine_kernel(const void* __restrict__ recv,
                                                           const uint32_t* __restrict__ flags, int world,
                                                           int64_t n, uint32_t epoch, void* __restrict__ y,
                                                           int* err) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int w = 0; w < world && ok; ++w) {
      if ((int32_t)(ld_acquire_sys(flags + w) - epoch) >= 0) continue;
      const uint64_t t0 = global_timer_ns();
      for (;;) {
        if ((int32_t)(ld_acquire_sys(flags + w) - epoch) >= 0) break;
        if (aborted(err) || global_timer_ns() - t0 > FP_WAIT_LIMIT_NS) {
          record_error(err, kErrPeerWait);
          ok = false;
          break;
        }
        __nanosleep(256);
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  __threadfence();
  const int64_t nv = n / 8;  // n % 8 == 0 (D % 64 == 0)
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    for (int w = 0; w < world; ++w) {
      if constexpr (kInF32) {
        const float4* p = reinterpret_cast<const float4*>(recv) + ((int64_t)w * n) / 4 + 2 * i;
        const float4 a = __ldcg(p), b = __ldcg(p + 1);
        acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
        acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
      } else {
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(recv) + ((int64_t)w * n) / 8 + i);
        const uint32_t ww[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          acc[2 * e] += __uint_as_float(ww[e] << 16);
          acc[2 * e + 1] += __uint_as_float(ww[e] & 0xFFFF0000u);
        }
      }
    }
    if constexpr (kOutF32) {
      float4* o = reinterpret_cast<float4*>(y) + 2 * i;
      o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    } else {
      uint32_t pk[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 b2 = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
        pk[e] = *reinterpret_cast<const uint32_t*>(&b2);
      }
      reinterpret_cast<uint4*>(y)[i] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  }
}

// The same `bytes` (a multiple of 16) from src to every destination (one 16-byte word per thread and
// destination per step): a rank's rows of a table every rank holds, written straight into the others'
// copies over NVLink.
__global__ void __launch_bounds__(256) peer_put_kernel(const uint4* __restrict__ src, int64_t words, PeerFlags dst) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < words; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 v = __ldg(src + i);
    for (int w = 0; w < dst.world; ++w) reinterpret_cast<uint4*>(dst.flag[w])[i] = v;
  }
}

// One thread waits (bounded) until every flag reached `epoch`; later work of the stream is ordered after it.
__global__ void peer_wait_kernel(const uint32_t* __restrict__ flags, int world, uint32_t epoch, int* err) {
  if (threadIdx.x != 0) return;
  for (int w = 0; w < world; ++w) {
    if ((int32_t)(ld_acquire_sys(flags + w) - epoch) >= 0) continue;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
      if ((int32_t)(ld_acquire_sys(flags + w) - epoch) >= 0) break;
      if (global_timer_ns() - t0 > FP_WAIT_LIMIT_NS) {
        record_error(err, kErrPeerWait);
        return;
      }
      __nanosleep(128);
    }
  }
  __threadfence();
}

int launch_peer_signal(const PeerFlags& f, uint32_t epoch, cudaStream_t st) {
  if (f.world < 1 || f.world > kMaxPeers) return FP_ERR_INVALID_ARG;
  peer_signal_kernel<<<1, 32, 0, st>>>(f, epoch);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

}  // namespace fp

using namespace fp;

extern "C" {

int fp_peer_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return FP_ERR_INVALID_ARG;
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return FP_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return FP_ERR_CUDA;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) <= FP_PEER_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return FP_OK;
}

int fp_peer_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return FP_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

int fp_peer_close(void* ptr) {
  if (!ptr) return FP_ERR_INVALID_ARG;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

int fp_peer_free(void* ptr) {
  if (!ptr) return FP_ERR_INVALID_ARG;
  return cudaFree(ptr) == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

int fp_peer_put(const void* src, size_t bytes, void* const* dst, int world, void* stream) {
  if (!src || !dst || world < 1 || world > kMaxPeers || bytes % 16) return FP_ERR_INVALID_ARG;
  PeerFlags d{};  // destinations (the flag slots hold the row pointers here)
  for (int w = 0; w < world; ++w) {
    if (!dst[w] || (reinterpret_cast<uintptr_t>(dst[w]) & 15u)) return FP_ERR_INVALID_ARG;
    d.flag[w] = static_cast<uint32_t*>(dst[w]);
  }
  d.world = world;
  if ((reinterpret_cast<uintptr_t>(src) & 15u)) return FP_ERR_INVALID_ARG;
  const int64_t words = (int64_t)(bytes / 16);
  if (words == 0) return FP_OK;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((words + 255) / 256, 148 * 2));
  peer_put_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(static_cast<const uint4*>(src), words, d);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

int fp_peer_signal(uint32_t* const* flags, int world, uint32_t epoch, void* stream) {
  if (!flags || world < 1 || world > kMaxPeers) return FP_ERR_INVALID_ARG;
  PeerFlags f{};
  for (int w = 0; w < world; ++w) {
    if (!flags[w]) return FP_ERR_INVALID_ARG;
    f.flag[w] = flags[w];
  }
  f.world = world;
  return launch_peer_signal(f, epoch, (cudaStream_t)stream);
}

int fp_peer_wait(const uint32_t* flags, int world, uint32_t epoch, void* workspace, size_t workspace_bytes,
                 void* stream) {
  if (!flags || !workspace || world < 1 || world > kMaxPeers) return FP_ERR_INVALID_ARG;
  if (workspace_bytes < 256) return FP_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(workspace, 0, 256, st) != cudaSuccess) return FP_ERR_CUDA;
  peer_wait_kernel<<<1, 32, 0, st>>>(flags, world, epoch, static_cast<int*>(workspace));
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

int fp_peer_combine(const void* recv, const uint32_t* flags, int world, int64_t rows, int D, int in_f32,
                    uint32_t epoch, void* y, int y_f32, void* workspace, size_t workspace_bytes, void* stream) {
  if (!recv || !flags || !y || !workspace || world < 1 || world > kMaxPeers || rows < 0 || D <= 0 || D % 8)
    return FP_ERR_INVALID_ARG;
  if (workspace_bytes < 256) return FP_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(recv) | reinterpret_cast<uintptr_t>(y)) & 15u) return FP_ERR_INVALID_ARG;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return FP_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  int* err = static_cast<int*>(workspace);
  if (cudaMemsetAsync(err, 0, 256, st) != cudaSuccess) return FP_ERR_CUDA;
  const int64_t n = rows * D;
  if (n == 0) return FP_OK;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n / 8 + 255) / 256, (int64_t)sms * 4));
  if (in_f32 && y_f32)
    peer_combine_kernel<true, true><<<grid, 256, 0, st>>>(recv, flags, world, n, epoch, y, err);
  else if (in_f32)
    peer_combine_kernel<true, false><<<grid, 256, 0, st>>>(recv, flags, world, n, epoch, y, err);
  else if (y_f32)
    peer_combine_kernel<false, true><<<grid, 256, 0, st>>>(recv, flags, world, n, epoch, y, err);
  else
    peer_combine_kernel<false, false><<<grid, 256, 0, st>>>(recv, flags, world, n, epoch, y, err);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

}  // extern "C"
