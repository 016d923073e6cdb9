// CUDA-core (FFMA) path of the Pattention contraction.
//
// Used for fp32 models, where the 1e-4 relative tolerance rules out tensor-core bf16/tf32 math, and for
// bf16 shapes the tensor-core kernels do not tile (widths not multiples of 64).  One CTA per token: for
// each active block b of the token,
//     g = x . K_gate[b]^T, u = x . K_up[b]^T (64 each; u only for SwiGLU), h = act(g, u), y += h . V[b]
// then y += ctx16 . W_out^T (additive stream) when requested.  y has D_out columns (v's width).
// Reference: foveal_indexer/pattention_triton.py:280-311 (per-token / shared-list fallback, all five
//            activations), foveal_indexer/foveal_pattention.py:329-342.
#include "fp_internal.cuh"

namespace fp {

constexpr int kSimtThreads = 256;

template <typename T>
__device__ __forceinline__ void store_out(void* y, int64_t i, float v, int y_f32) {
  if (y_f32) reinterpret_cast<float*>(y)[i] = v;
  else reinterpret_cast<T*>(y)[i] = (T)v;
}
template <>
__device__ __forceinline__ void store_out<__nv_bfloat16>(void* y, int64_t i, float v, int y_f32) {
  if (y_f32) reinterpret_cast<float*>(y)[i] = v;
  else reinterpret_cast<__nv_bfloat16*>(y)[i] = __float2bfloat16_rn(v);
}

template <typename T, int CPT>
__global__ void __launch_bounds__(kSimtThreads)
simt_pattention_kernel(const SimtArgs a) {
  extern __shared__ float sh[];  // x row [D] fp32, then gu [128]
  float* xs = sh;
  float* gu = sh + a.D;
  const int D = a.D;
  const int Do = a.D_out > 0 ? a.D_out : a.D;
  const bool gated = a.act == FP_ACT_SWIGLU;
  const int64_t t = blockIdx.x;
  const T* x = reinterpret_cast<const T*>(a.x) + t * D;
  const T* kg = reinterpret_cast<const T*>(a.k_gate);
  const T* ku = reinterpret_cast<const T*>(a.k_up);
  const T* v = reinterpret_cast<const T*>(a.v);
  for (int d = threadIdx.x; d < D; d += kSimtThreads) xs[d] = to_f32(x[d]);

  float acc[CPT];
#pragma unroll
  for (int i = 0; i < CPT; ++i) acc[i] = 0.f;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int n_list;
  if (a.active) n_list = a.n_active;
  else n_list = a.base + a.rcnt[t];
  __syncthreads();

  for (int li = 0; li < n_list; ++li) {
    int b;
    if (a.active) b = a.active[li];
    else b = li < a.base ? li : a.ridx[t * a.cap + (li - a.base)];
    if (!a.active && (b % a.stride) != a.offset) continue;
    if (b < 0 || b >= a.NB) continue;
    // 128 dot products: warp w computes rows 16w .. 16w+15 of [gate(64); up(64)]
    for (int r = warp * 16; r < warp * 16 + 16; ++r) {
      if (!gated && r >= 64) break;  // non-gated forms need the gate rows only
      const T* wrow = (r < 64 ? kg + ((int64_t)b * 64 + r) * D : ku + ((int64_t)b * 64 + r - 64) * D);
      float s = 0.f;
      for (int d = lane; d < D; d += 32) s = fmaf(xs[d], to_f32(wrow[d]), s);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) gu[r] = s;
    }
    __syncthreads();
    if (threadIdx.x < 64) {
      const float g = gu[threadIdx.x];
      gu[threadIdx.x] = pattention_act<true>(a.act, g, gated ? gu[64 + threadIdx.x] : 0.0f);
    }
    __syncthreads();
    const T* vb = v + (int64_t)b * 64 * Do;
#pragma unroll
    for (int i = 0; i < CPT; ++i) {
      const int d = threadIdx.x + i * kSimtThreads;
      if (d < Do) {
        float s = acc[i];
        for (int j = 0; j < 64; ++j) s = fmaf(gu[j], to_f32(vb[(int64_t)j * Do + d]), s);
        acc[i] = s;
      }
    }
    __syncthreads();
  }

  float ctx[16];
  if (a.ctx16) {
#pragma unroll
    for (int k = 0; k < 16; ++k) ctx[k] = a.ctx16[t * 16 + k];
  }
  const T* wo = reinterpret_cast<const T*>(a.out_proj);
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int d = threadIdx.x + i * kSimtThreads;
    if (d < Do) {
      float o = acc[i];
      if (a.ctx16) {
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) s = fmaf(ctx[k], to_f32(wo[(int64_t)d * 16 + k]), s);
        o += s;
      }
      store_out<T>(a.y, t * Do + d, o, a.y_f32);
    }
  }
}

template <typename T>
static int launch_simt_t(const SimtArgs& a, cudaStream_t st) {
  const size_t smem = ((size_t)a.D + 128) * sizeof(float);
  const int cpt = ((a.D_out > 0 ? a.D_out : a.D) + kSimtThreads - 1) / kSimtThreads;
  auto go = [&](auto kern) -> int {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return FP_ERR_CUDA;
    kern<<<(unsigned)a.M, kSimtThreads, smem, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
  };
  if (cpt <= 1) return go(simt_pattention_kernel<T, 1>);
  if (cpt <= 2) return go(simt_pattention_kernel<T, 2>);
  if (cpt <= 4) return go(simt_pattention_kernel<T, 4>);
  if (cpt <= 8) return go(simt_pattention_kernel<T, 8>);
  if (cpt <= 16) return go(simt_pattention_kernel<T, 16>);
  if (cpt <= 32) return go(simt_pattention_kernel<T, 32>);
  return FP_ERR_UNSUPPORTED;
}

int launch_simt(const SimtArgs& a, cudaStream_t st) {
  if (a.M <= 0) return FP_OK;
  return a.dtype == FP_DTYPE_BF16 ? launch_simt_t<__nv_bfloat16>(a, st) : launch_simt_t<float>(a, st);
}

}  // namespace fp
