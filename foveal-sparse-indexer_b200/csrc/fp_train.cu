// Training-mode pieces: the fused SwiGLU backward of the active-set contraction.
//
// Reference: TritonFusedSwiGLUFunction.backward / _swiglu_bwd_kernel (foveal_indexer/pattention_triton.py:49-96):
//   sig = sigmoid(g), silu = g * sig
//   du = dout * silu,  dg = dout * u * sig * (1 + g * (1 - sig))
// computed in fp32 from inputs of the GEMM dtype, stored in that dtype.  The activation itself,
// h = silu * u (needed for the gradient of v), comes out of the same pass.
#include "fp_internal.cuh"

namespace fp {
namespace {

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename T>
__global__ void swiglu_bwd_kernel(const T* __restrict__ dout, const T* __restrict__ g, const T* __restrict__ u,
                                  int64_t n, T* __restrict__ dg, T* __restrict__ du, T* __restrict__ h) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float d = to_f32(dout[i]), gv = to_f32(g[i]), uv = to_f32(u[i]);
    const float sig = 1.0f / (1.0f + expf(-gv));
    const float silu = gv * sig;
    du[i] = from_f32<T>(d * silu);
    dg[i] = from_f32<T>(d * uv * (sig * (1.0f + gv * (1.0f - sig))));
    if (h) h[i] = from_f32<T>(silu * uv);
  }
}

}  // namespace
}  // namespace fp

using namespace fp;

extern "C" {

int fp_swiglu_bwd(const void* dout, const void* g, const void* u, int dtype, int64_t n, void* dg, void* du, void* h,
                  void* stream) {
  if (n < 0) return FP_ERR_INVALID_ARG;
  if (n == 0) return FP_OK;
  if (!dout || !g || !u || !dg || !du) return FP_ERR_INVALID_ARG;
  if (dtype != FP_DTYPE_F32 && dtype != FP_DTYPE_BF16) return FP_ERR_UNSUPPORTED;
  (void)cudaGetLastError();
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return FP_ERR_CUDA;
  const int64_t want = (n + 255) / 256;
  const int blocks = (int)(want < (int64_t)sms * 16 ? want : (int64_t)sms * 16);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == FP_DTYPE_BF16)
    swiglu_bwd_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        (const __nv_bfloat16*)dout, (const __nv_bfloat16*)g, (const __nv_bfloat16*)u, n, (__nv_bfloat16*)dg,
        (__nv_bfloat16*)du, (__nv_bfloat16*)h);
  else
    swiglu_bwd_kernel<float><<<blocks, 256, 0, st>>>((const float*)dout, (const float*)g, (const float*)u, n,
                                                     (float*)dg, (float*)du, (float*)h);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

}  // extern "C"
