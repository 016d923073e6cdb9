// Elementwise SwiGLU: the forward of triton_fused_swiglu (h = silu(g) * u, pattention_triton.py:30-47) and
// the fused backward of the active-set contraction.
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

// h = silu(g) * u in fp32 (exact expf and division, like the backward), stored in the input dtype.  bf16
// runs of 8 elements move as 16-byte words when the pointers and n allow it.
template <typename T>
__global__ void swiglu_fwd_kernel(const T* __restrict__ g, const T* __restrict__ u, int64_t n, T* __restrict__ h) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float gv = to_f32(g[i]);
    h[i] = from_f32<T>(gv / (1.0f + expf(-gv)) * to_f32(u[i]));
  }
}

__global__ void swiglu_fwd_bf16x8_kernel(const uint4* __restrict__ g, const uint4* __restrict__ u, int64_t n8,
                                         uint4* __restrict__ h) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 gw = g[i], uw = u[i];
    const uint32_t ga[4] = {gw.x, gw.y, gw.z, gw.w}, ua[4] = {uw.x, uw.y, uw.z, uw.w};
    uint32_t out[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float g0 = __uint_as_float(ga[k] << 16), g1 = __uint_as_float(ga[k] & 0xFFFF0000u);
      const float u0 = __uint_as_float(ua[k] << 16), u1 = __uint_as_float(ua[k] & 0xFFFF0000u);
      const __nv_bfloat162 r = __floats2bfloat162_rn(g0 / (1.0f + expf(-g0)) * u0, g1 / (1.0f + expf(-g1)) * u1);
      out[k] = *reinterpret_cast<const uint32_t*>(&r);
    }
    h[i] = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

int grid_for(int64_t n) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return -1;
  const int64_t want = (n + 255) / 256;
  return (int)(want < (int64_t)sms * 16 ? want : (int64_t)sms * 16);
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

int fp_swiglu_fwd(const void* g, const void* u, int dtype, int64_t n, void* h, void* stream) {
  if (n < 0) return FP_ERR_INVALID_ARG;
  if (n == 0) return FP_OK;
  if (!g || !u || !h) return FP_ERR_INVALID_ARG;
  if (dtype != FP_DTYPE_F32 && dtype != FP_DTYPE_BF16) return FP_ERR_UNSUPPORTED;
  (void)cudaGetLastError();
  cudaStream_t st = (cudaStream_t)stream;
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (dtype == FP_DTYPE_BF16 && n % 8 == 0 && al16(g) && al16(u) && al16(h)) {
    const int blocks = grid_for(n / 8);
    if (blocks < 0) return FP_ERR_CUDA;
    swiglu_fwd_bf16x8_kernel<<<blocks, 256, 0, st>>>((const uint4*)g, (const uint4*)u, n / 8, (uint4*)h);
  } else {
    const int blocks = grid_for(n);
    if (blocks < 0) return FP_ERR_CUDA;
    if (dtype == FP_DTYPE_BF16)
      swiglu_fwd_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>((const __nv_bfloat16*)g, (const __nv_bfloat16*)u, n,
                                                              (__nv_bfloat16*)h);
    else
      swiglu_fwd_kernel<float><<<blocks, 256, 0, st>>>((const float*)g, (const float*)u, n, (float*)h);
  }
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

}  // extern "C"
