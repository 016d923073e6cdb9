// Kernels of the layers that share the 16-D router with the Pattention MLP but contract over the UNION of
// the blocks the call's tokens selected: BlockSparseLinear (foveal_indexer/block_matmul.py:129-282) and
// FovealTokenformerLinear (foveal_indexer/tokenformer.py:132-228).
//
//   param_blocks_16d   pooled 16-D key / value per 64-row block of a parameter matrix
//                      (FovealIndexer.compute_kv_blocks_16d core.py:225-252; BlockSparseLinear.
//                      get_block_keys_and_values block_matmul.py:107-127)
//   union              ascending ids of the base blocks and every selected remote block, then the
//                      unselected ids (block_matmul.py:206-217; tokenformer.py:171-181); the count stays
//                      on the device so that the contractions that follow need no host round trip
//   rowact             Tokenformer activation over the active parameter tokens of a row: softmax(s / c)
//                      or gelu(s / ||s||_2) (tokenformer.py:101-110)
//   fill_inactive      BlockSparseLinear output columns of unselected blocks: the additive stream only
//                      (block_matmul.py:240-254)
//   mapped_gemm_simt   CUDA-core contraction over mapped 64-wide blocks, for fp32 layers (the 1e-4
//                      tolerance of fp32 rules out bf16/tf32 tensor cores) and untileable shapes; the
//                      bf16 tensor-core form is the block-mapped down kernel of fp_gemm.cu
//   transpose          v -> v_t (fp_pack_weights) and v_param -> v_param^T: the K-major operands of the
//                      tensor-core contractions
#include "fp_internal.cuh"

#include <algorithm>

namespace fp {

// ---------------------------------------------------------------- block reductions (256 threads)
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w];  // fixed order on every thread
  return s;
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = -INFINITY;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
  return m;
}

// ---------------------------------------------------------------- pooled 16-D keys / values
// One CTA per block of 64 rows; warp w projects rows w, w + 8, ... onto the 16 key and 16 value
// directions (lane-strided dot products, butterfly-reduced), rms-normalises the key projection
// (eps = fp32 machine epsilon, F.rms_norm's default), then 32 threads average over the 64 rows in row
// order and the key mean is L2-normalised (F.normalize: divided by max(||k||, 1e-12)).
template <typename T>
__global__ void __launch_bounds__(256) param_blocks_kernel(const T* __restrict__ P, const T* __restrict__ wk,
                                                           const T* __restrict__ wv, int D, float* __restrict__ kb,
                                                           float* __restrict__ vb) {
  __shared__ float ke[64][16];
  __shared__ float ve[64][16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t b = blockIdx.x;
  for (int rr = warp; rr < 64; rr += 8) {
    const T* prow = P + (b * 64 + rr) * (int64_t)D;
    float acc[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[j] = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float xv = to_f32(prow[d]);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        acc[j] = fmaf(xv, to_f32(wk[(int64_t)j * D + d]), acc[j]);
        acc[16 + j] = fmaf(xv, to_f32(wv[(int64_t)j * D + d]), acc[16 + j]);
      }
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    }
    if (lane == 0) {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) ss = fmaf(acc[j], acc[j], ss);
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(ss * (1.0f / 16.0f) + 1.1920928955078125e-07f));
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        ke[rr][j] = acc[j] * inv;
        ve[rr][j] = acc[16 + j];
      }
    }
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int j = threadIdx.x & 15;
    const bool isv = threadIdx.x >= 16;
    float s = 0.f;
    for (int r = 0; r < 64; ++r) s += isv ? ve[r][j] : ke[r][j];
    s = s * (1.0f / 64.0f);
    float ss = s * s;  // lanes 0-15 and 16-31 reduce separately
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (isv) vb[b * 16 + j] = s;
    else kb[b * 16 + j] = __fdiv_rn(s, fmaxf(__fsqrt_rn(ss), 1e-12f));
  }
}

int launch_param_blocks_16d(const void* P, const void* wk, const void* wv, int dtype, int64_t N, int D,
                            float* kb, float* vb, cudaStream_t st) {
  const int64_t nb = N / 64;
  if (nb <= 0) return FP_OK;
  if (dtype == FP_DTYPE_BF16)
    param_blocks_kernel<__nv_bfloat16><<<(unsigned)nb, 256, 0, st>>>(
        (const __nv_bfloat16*)P, (const __nv_bfloat16*)wk, (const __nv_bfloat16*)wv, D, kb, vb);
  else
    param_blocks_kernel<float><<<(unsigned)nb, 256, 0, st>>>((const float*)P, (const float*)wk,
                                                             (const float*)wv, D, kb, vb);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

// ---------------------------------------------------------------- union of the selected blocks
__global__ void union_mark_kernel(const int32_t* __restrict__ idx, const int32_t* __restrict__ cnt, int64_t M,
                                  int cap, int NB, int base, int32_t* __restrict__ flags) {
  const int64_t n = M * cap;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / cap;
    const int k = (int)(i - t * cap);
    if (k < min(cnt[t], cap)) {
      const int b = idx[i];
      if (b >= base && b < NB) flags[b] = 1;  // every writer stores the same value
    }
  }
}

constexpr int kUnionThreads = 1024;
constexpr int kUnionMaxBlocks = 8192;

// blocks[] holds flags on entry; on exit blocks[0..n) = selected ids ascending, blocks[n..NB) = the
// others ascending, *n_active = n.  Every flag is read into shared memory before any write.
__global__ void __launch_bounds__(kUnionThreads) union_compact_kernel(int32_t* __restrict__ blocks, int NB, int base,
                                                                      int32_t* __restrict__ n_active) {
  __shared__ uint8_t fl[kUnionMaxBlocks];
  __shared__ int wsum[kUnionThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int b = tid; b < NB; b += kUnionThreads) fl[b] = (b < base || blocks[b] != 0) ? 1 : 0;
  __syncthreads();
  const int E = (NB + kUnionThreads - 1) / kUnionThreads;
  const int s0 = tid * E;
  int mine = 0;
  for (int e = 0; e < E; ++e)
    if (s0 + e < NB) mine += fl[s0 + e];
  int incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int up = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += up;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  int before = 0, total = 0;
  for (int w = 0; w < kUnionThreads / 32; ++w) {
    before += w < warp ? wsum[w] : 0;
    total += wsum[w];
  }
  const int excl = before + incl - mine;
  int pa = excl, pi = total + (s0 < NB ? s0 : NB) - excl;
  for (int e = 0; e < E; ++e) {
    const int b = s0 + e;
    if (b < NB) {
      if (fl[b]) blocks[pa++] = b;
      else blocks[pi++] = b;
    }
  }
  if (tid == 0) *n_active = total;
}

int launch_union(const int32_t* idx, const int32_t* cnt, int64_t M, int capacity, int NB, int base,
                 int32_t* active, int32_t* n_active, cudaStream_t st) {
  if (NB <= 0 || NB > kUnionMaxBlocks) return FP_ERR_UNSUPPORTED;
  if (cudaMemsetAsync(active, 0, (size_t)NB * sizeof(int32_t), st) != cudaSuccess) return FP_ERR_CUDA;
  const int64_t n = M * capacity;
  if (n > 0) {
    const int blocks = (int)std::min<int64_t>((n + 255) / 256, 4096);
    union_mark_kernel<<<blocks, 256, 0, st>>>(idx, cnt, M, capacity, NB, base, active);
    if (cudaGetLastError() != cudaSuccess) return FP_ERR_CUDA;
  }
  union_compact_kernel<<<1, kUnionThreads, 0, st>>>(active, NB, base, n_active);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

// ---------------------------------------------------------------- Tokenformer activation
// Row m of S [M, lds] (fp32 raw scores x . k_param^T of the active parameter tokens, in union order)
// -> P [M, ldp] over the first 64 * n_active columns.  mode 0: softmax(s / div); mode 1:
// gelu(s / max(||s||_2, 1e-12)) with the exact (erf) GELU.
__device__ __forceinline__ float ld_score(const float* p, int c) { return p[c]; }
__device__ __forceinline__ float ld_score(const __nv_bfloat16* p, int c) { return __bfloat162float(p[c]); }

template <typename InT, typename OutT>
__global__ void __launch_bounds__(256) rowact_kernel(const InT* __restrict__ S, int64_t lds,
                                                     const int32_t* __restrict__ n_active, int mode, float div,
                                                     OutT* __restrict__ P, int64_t ldp) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int n = (int)min((int64_t)*n_active * 64, lds);  // never past the row
  const InT* s = S + row * lds;
  OutT* p = P + row * ldp;
  if (mode == 0) {
    float mx = -INFINITY;
    for (int c = threadIdx.x; c < n; c += blockDim.x) mx = fmaxf(mx, __fdiv_rn(ld_score(s, c), div));
    mx = block_max(mx, red);
    float sum = 0.f;
    for (int c = threadIdx.x; c < n; c += blockDim.x) sum += expf(__fdiv_rn(ld_score(s, c), div) - mx);
    sum = block_sum(sum, red);
    for (int c = threadIdx.x; c < n; c += blockDim.x) {
      const float v = __fdiv_rn(expf(__fdiv_rn(ld_score(s, c), div) - mx), sum);
      p[c] = (OutT)v;
    }
  } else {
    float ss = 0.f;
    for (int c = threadIdx.x; c < n; c += blockDim.x) ss = fmaf(ld_score(s, c), ld_score(s, c), ss);
    ss = block_sum(ss, red);
    const float nrm = fmaxf(__fsqrt_rn(ss), 1e-12f);
    for (int c = threadIdx.x; c < n; c += blockDim.x) {
      const float u = __fdiv_rn(ld_score(s, c), nrm);
      p[c] = (OutT)(u * 0.5f * (1.0f + erff(u * 0.70710678118654752440f)));
    }
  }
}

// Single-pass form for rows of at most 256 * EPT active columns: the row is read once into registers
// (element i * 256 + thread of each thread), reduced, and written; same arithmetic as rowact_kernel.
template <typename InT, typename OutT, int EPT>
__global__ void __launch_bounds__(256) rowact_reg_kernel(const InT* __restrict__ S, int64_t lds,
                                                         const int32_t* __restrict__ n_active, int mode, float div,
                                                         OutT* __restrict__ P, int64_t ldp) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int n = (int)min(min((int64_t)*n_active * 64, lds), (int64_t)256 * EPT);  // never past the row
  const InT* s = S + row * lds;
  OutT* p = P + row * ldp;
  float v[EPT];
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    const int c = i * 256 + threadIdx.x;
    v[i] = c < n ? ld_score(s, c) : 0.f;
  }
  // The per-row divisors (sqrt(D_in), the exponential sum, the row norm) are applied as one reciprocal
  // and a multiply per element (within one rounding of a division); the kernel is otherwise bound by
  // the issue of IEEE divisions rather than by its memory traffic.
  if (mode == 0) {
    const float inv_div = __frcp_rn(div);
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      if (i * 256 + (int)threadIdx.x < n) {
        v[i] *= inv_div;
        mx = fmaxf(mx, v[i]);
      }
    }
    mx = block_max(mx, red);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      if (i * 256 + (int)threadIdx.x < n) {
        v[i] = expf(v[i] - mx);
        sum += v[i];
      }
    }
    sum = block_sum(sum, red);
    const float inv_sum = __frcp_rn(sum);
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int c = i * 256 + threadIdx.x;
      if (c < n) p[c] = (OutT)(v[i] * inv_sum);
    }
  } else {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < EPT; ++i) ss = fmaf(v[i], v[i], ss);  // zero beyond n
    ss = block_sum(ss, red);
    const float inv_nrm = __frcp_rn(fmaxf(__fsqrt_rn(ss), 1e-12f));
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int c = i * 256 + threadIdx.x;
      if (c < n) {
        const float u = v[i] * inv_nrm;
        p[c] = (OutT)(u * 0.5f * (1.0f + erff(u * 0.70710678118654752440f)));
      }
    }
  }
}

// max_cols: an upper bound of 64 * n_active (the parameter-token count), known on the host.  S is fp32, or
// bf16 (s_bf16) on the tensor-core path, where the scores are rounded to bf16 as the reference's bf16
// layer rounds its raw scores.
int launch_rowact(const void* S, int s_bf16, int64_t lds, int64_t M, const int32_t* n_active, int mode, float div,
                  void* P, int64_t ldp, int p_f32, cudaStream_t st, int max_cols) {
  if (M <= 0) return FP_OK;
  if (M > INT32_MAX) return FP_ERR_UNSUPPORTED;
  auto go = [&](auto in_tag, auto out_tag) -> int {
    using InT = decltype(in_tag);
    using OutT = decltype(out_tag);
    const InT* St = static_cast<const InT*>(S);
    OutT* Pt = static_cast<OutT*>(P);
    const unsigned g = (unsigned)M;
    if (max_cols <= 256 * 4) rowact_reg_kernel<InT, OutT, 4><<<g, 256, 0, st>>>(St, lds, n_active, mode, div, Pt, ldp);
    else if (max_cols <= 256 * 8) rowact_reg_kernel<InT, OutT, 8><<<g, 256, 0, st>>>(St, lds, n_active, mode, div, Pt, ldp);
    else if (max_cols <= 256 * 16) rowact_reg_kernel<InT, OutT, 16><<<g, 256, 0, st>>>(St, lds, n_active, mode, div, Pt, ldp);
    else if (max_cols <= 256 * 32) rowact_reg_kernel<InT, OutT, 32><<<g, 256, 0, st>>>(St, lds, n_active, mode, div, Pt, ldp);
    else rowact_kernel<InT, OutT><<<g, 256, 0, st>>>(St, lds, n_active, mode, div, Pt, ldp);
    return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
  };
  if (s_bf16) return p_f32 ? go(__nv_bfloat16{}, float{}) : go(__nv_bfloat16{}, __nv_bfloat16{});
  return p_f32 ? go(float{}, float{}) : go(float{}, __nv_bfloat16{});
}

// ---------------------------------------------------------------- BlockSparseLinear inactive columns
template <typename OutT, typename WT>
__global__ void fill_inactive_kernel(const int32_t* __restrict__ blocks, const int32_t* __restrict__ n_active, int NB,
                                     int64_t M, const float* __restrict__ ctx16, const WT* __restrict__ out_proj,
                                     OutT* __restrict__ out, int64_t ldo) {
  const int n = *n_active;
  const int64_t cols = (int64_t)(NB - n) * 64;
  const int64_t total = M * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / cols;
    const int cc = (int)(i - m * cols);
    const int blk = blocks[n + cc / 64];
    if ((unsigned)blk >= (unsigned)NB) continue;  // not a block of this layer (a corrupt list): skipped
    const int col = blk * 64 + cc % 64;
    float v = 0.f;
    if (ctx16) {
#pragma unroll
      for (int k = 0; k < 16; ++k) v = fmaf(ctx16[m * 16 + k], to_f32(out_proj[(int64_t)col * 16 + k]), v);
    }
    out[m * ldo + col] = (OutT)v;
  }
}

int launch_fill_inactive(const int32_t* blocks, const int32_t* n_active, int NB, int64_t M, const float* ctx16,
                         const void* out_proj, int dtype, void* out, int64_t ldo, int num_sms, cudaStream_t st) {
  if (M <= 0) return FP_OK;
  const int grid = std::max(1, num_sms) * 8;
  if (dtype == FP_DTYPE_BF16)
    fill_inactive_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, 256, 0, st>>>(
        blocks, n_active, NB, M, ctx16, (const __nv_bfloat16*)out_proj, (__nv_bfloat16*)out, ldo);
  else
    fill_inactive_kernel<float, float><<<grid, 256, 0, st>>>(blocks, n_active, NB, M, ctx16,
                                                             (const float*)out_proj, (float*)out, ldo);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

// ---------------------------------------------------------------- CUDA-core mapped contraction
// Y[m, col(c)] = sum_k A[m, k] . Bv(k, c) (+ bias[col(c)]) (+ ctx16[m] . out_proj[col(c)]^T)
//   nn = 0: Bv(k, c) = B[row(c) * ldb + k], row(c) = nmap[c / 64] * 64 + c % 64 (or c), c < ncols
//   nn = 1: Bv(k, c) = B[row(k) * ldb + c], row(k) = kmap[k / 64] * 64 + k % 64 (or k), k < kcols
//   col(c) = omap[c / 64] * 64 + c % 64 (or c)
// 64 x 64 output tile per CTA (one column block), 256 threads of 4 x 4 outputs, k-steps of 16 in
// shared memory; fp32 accumulation in k order.
__device__ __forceinline__ float ld_any(const void* p, int64_t i, int f32) {
  return f32 ? reinterpret_cast<const float*>(p)[i] : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

__global__ void __launch_bounds__(256) mapped_gemm_simt_kernel(const MappedGemm g) {
  __shared__ float As[16][64 + 1];
  __shared__ float Bs[16][64 + 1];
  const int ncols = g.ncnt ? min(*g.ncnt * 64, g.N) : g.N;
  const int kcols = g.kcnt ? min(*g.kcnt * 64, g.K) : g.K;
  const int c0 = blockIdx.x * 64;
  const int64_t m0 = (int64_t)blockIdx.y * 64;
  if (c0 >= ncols) return;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t brow_c = g.nn ? 0 : (g.nmap ? (int64_t)g.nmap[c0 / 64] * 64 : c0);  // nn = 0: B rows of this tile
  const int64_t ocol_c = g.omap ? (int64_t)g.omap[c0 / 64] * 64 : c0;               // Y columns of this tile
  // map entries outside B or Y (a corrupt block list) leave the tile untouched
  if ((g.nmap && !g.nn && (brow_c < 0 || brow_c + 64 > g.N)) || (g.omap && (ocol_c < 0 || ocol_c + 64 > g.ldy)))
    return;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < kcols; k0 += 16) {
    // A tile: 64 rows x 16 k
    for (int e = tid; e < 64 * 16; e += 256) {
      const int r = e / 16, kk = e % 16;
      const int64_t m = m0 + r;
      const int k = k0 + kk;
      As[kk][r] = (m < g.M && k < kcols) ? ld_any(g.a, m * g.lda + k, g.a_f32) : 0.f;
    }
    // B tile: 16 k x 64 columns
    for (int e = tid; e < 64 * 16; e += 256) {
      float v = 0.f;
      if (g.nn) {
        const int kk = e / 64, cc = e % 64;
        const int k = k0 + kk, c = c0 + cc;
        if (k < kcols && c < ncols) {
          const int64_t row = g.kmap ? (int64_t)g.kmap[k / 64] * 64 + k % 64 : k;
          if (row >= 0 && row < g.K) v = ld_any(g.b, row * g.ldb + c, g.b_f32);
        }
        Bs[kk][cc] = v;
      } else {
        const int cc = e / 16, kk = e % 16;
        const int k = k0 + kk, c = c0 + cc;
        if (k < kcols && c < ncols) v = ld_any(g.b, (brow_c + cc) * g.ldb + k, g.b_f32);
        Bs[kk][cc] = v;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty * 4 + i;
    if (m >= g.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = c0 + tx * 4 + j;
      if (c >= ncols) continue;
      const int64_t col = ocol_c + (c - c0);
      float v = acc[i][j];
      if (g.bias) v += ld_any(g.bias, col, g.bias_f32);
      if (g.ctx16) {
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) s = fmaf(g.ctx16[m * 16 + k], ld_any(g.out_proj, col * 16 + k, g.out_proj_f32), s);
        v += s;
      }
      if (g.y_f32) reinterpret_cast<float*>(g.y)[m * g.ldy + col] = v;
      else reinterpret_cast<__nv_bfloat16*>(g.y)[m * g.ldy + col] = __float2bfloat16_rn(v);
    }
  }
}

int launch_mapped_gemm_simt(const MappedGemm& g, cudaStream_t st) {
  if (g.M <= 0 || g.N <= 0) return FP_OK;
  const int64_t mt = (g.M + 63) / 64;
  if (mt > 65535) return FP_ERR_UNSUPPORTED;
  dim3 grid((unsigned)((g.N + 63) / 64), (unsigned)mt);
  mapped_gemm_simt_kernel<<<grid, 256, 0, st>>>(g);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

// ---------------------------------------------------------------- transpose (32 x 32 tiles)
template <typename T>
__global__ void transpose_kernel(const T* __restrict__ src, int64_t rows, int64_t cols, T* __restrict__ dst) {
  __shared__ T tile[32][33];
  const int64_t c0 = (int64_t)blockIdx.x * 32, r0 = (int64_t)blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = src[r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) dst[c * rows + r] = tile[threadIdx.x][i];
  }
}

int launch_transpose(const void* src, int64_t rows, int64_t cols, int dtype, void* dst, cudaStream_t st) {
  if (rows <= 0 || cols <= 0) return FP_OK;
  if ((rows + 31) / 32 > 65535) return FP_ERR_UNSUPPORTED;
  dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32)), block(32, 8);
  if (dtype == FP_DTYPE_BF16)
    transpose_kernel<__nv_bfloat16><<<grid, block, 0, st>>>((const __nv_bfloat16*)src, rows, cols, (__nv_bfloat16*)dst);
  else
    transpose_kernel<float><<<grid, block, 0, st>>>((const float*)src, rows, cols, (float*)dst);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

}  // namespace fp
