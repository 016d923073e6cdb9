// 16-D foveal router, top-p block selection, block-CSR construction and pooled routing.
//
// Reference semantics (kreasof-ai/foveal-sparse-indexer):
//   compute_router_scores   foveal_indexer/foveal_pattention.py:257-262
//   masked_softmax          foveal_indexer/core.py:36-43
//   select_blocks           foveal_indexer/core.py:46-160 (non-causal branch :90-99)
//   pooled routing          foveal_indexer/foveal_pattention.py:292-303 (train), :310-321 (eval)
//   additive-stream context foveal_indexer/foveal_pattention.py:338-340
//
// All router arithmetic is fp32 (the cumulative sum accumulates in fp64 and rounds every prefix to
// fp32, as PyTorch's CPU cumsum does).  Ties in probability are broken toward the lower block id.
#include "fp_internal.cuh"

#include <algorithm>

namespace fp {

// --------------------------------------------------------------------------------------------
// Scores: S[m, b] = (rms_norm(x[m] . Wq^T) . K16[b]) / sqrt(16)  [/ temperature]
// One warp handles TPW tokens at a time; lanes split the hidden dimension in 8-element vectors.
// --------------------------------------------------------------------------------------------
constexpr int kScoreTPW = 4;
constexpr int kScoreWarps = 8;

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

template <typename T>
__global__ void __launch_bounds__(kScoreWarps * 32)
router_scores_kernel(const T* __restrict__ x, const T* __restrict__ wq, const T* __restrict__ k16,
                     int64_t M, int D, int NB, float inv_scale_div, float temperature,
                     float* __restrict__ scores, float* __restrict__ q16_out) {
  extern __shared__ float sk[];  // [16][NB] fp32 block keys, transposed: lanes read consecutive blocks
  for (int i = threadIdx.x; i < NB * 16; i += blockDim.x) sk[(i & 15) * NB + (i >> 4)] = to_f32(k16[i]);
  __syncthreads();

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t tok0 = ((int64_t)blockIdx.x * kScoreWarps + warp) * kScoreTPW;
  if (tok0 >= M) return;

  float acc[kScoreTPW][16];
#pragma unroll
  for (int t = 0; t < kScoreTPW; ++t)
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[t][j] = 0.f;

  for (int c = lane * 8; c < D; c += 256) {
    float xv[kScoreTPW][8];
#pragma unroll
    for (int t = 0; t < kScoreTPW; ++t) {
      const int64_t tok = tok0 + t < M ? tok0 + t : M - 1;
      load8<T>(x + tok * D + c, xv[t]);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float wv[8];
      load8<T>(wq + (int64_t)j * D + c, wv);
#pragma unroll
      for (int t = 0; t < kScoreTPW; ++t)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[t][j] = fmaf(xv[t][e], wv[e], acc[t][j]);
    }
  }
#pragma unroll
  for (int t = 0; t < kScoreTPW; ++t)
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float v = acc[t][j];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[t][j] = v;
    }

  const float eps = 1.1920928955078125e-07f;  // torch.finfo(float32).eps: F.rms_norm's default
#pragma unroll
  for (int t = 0; t < kScoreTPW; ++t) {
    const int64_t tok = tok0 + t;
    if (tok >= M) break;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) ss = fmaf(acc[t][j], acc[t][j], ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(ss * (1.0f / 16.0f) + eps));
    float q[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) q[j] = acc[t][j] * inv;
    if (q16_out && lane < 16) {
      float qv = q[0];
#pragma unroll
      for (int j = 1; j < 16; ++j) qv = (lane == j) ? q[j] : qv;
      q16_out[tok * 16 + lane] = qv;
    }
    for (int b = lane; b < NB; b += 32) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) s = fmaf(q[j], sk[j * NB + b], s);
      s = s * inv_scale_div;            // / sqrt(16): exact power-of-two scaling
      if (temperature != 1.0f) s = __fdiv_rn(s, temperature);
      scores[tok * NB + b] = s;
    }
  }
}

// --------------------------------------------------------------------------------------------
// bf16 scores with tensor-core MMA (mma.sync m16n8k16, fp32 accumulate).  One warp computes the 16
// projections of 16 tokens.  The contraction index is permuted inside each 64-element chunk so that
// every lane reads contiguous 32-byte pieces of x and W_q: lane (g, t) of k-step s uses elements
// 16t + 4s + {0..3}, which is where the fragment layout wants columns {2t, 2t+1, 2t+8, 2t+9} of
// that step; A and B share the permutation, so the sum is unchanged.
// --------------------------------------------------------------------------------------------
constexpr int kMmaWarps = 4;

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ld32B(const __nv_bfloat16* p, uint32_t (&w)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(p) + 1);
  w[0] = u.x; w[1] = u.y; w[2] = u.z; w[3] = u.w; w[4] = v.x; w[5] = v.y; w[6] = v.z; w[7] = v.w;
}

// One CTA of kMmaWarps warps per 16 tokens: warp w accumulates the D-range [w*D/4, (w+1)*D/4) (four
// times the memory-level parallelism of one warp per group), partial projections are summed in
// shared memory, then each warp finishes 4 of the 16 tokens (RMSNorm, 16-D scores).
__global__ void __launch_bounds__(kMmaWarps * 32)
router_scores_mma_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ wq,
                         const __nv_bfloat16* __restrict__ k16, int64_t M, int D, int NB,
                         float* __restrict__ scores, float* __restrict__ q16_out) {
  extern __shared__ float sk[];  // [16][NB] transposed block keys, then [kMmaWarps][16][17] partials
  float* sq = sk + 16 * NB;
  for (int i = threadIdx.x; i < NB * 16; i += blockDim.x) sk[(i & 15) * NB + (i >> 4)] = __bfloat162float(k16[i]);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int64_t tok0 = (int64_t)blockIdx.x * 16;
  const int dpart = D / kMmaWarps;  // multiple of 64 (D % 256 == 0)
  const int kbeg = warp * dpart;
  const __nv_bfloat16* xa = x + (tok0 + g < M ? tok0 + g : M - 1) * (int64_t)D + kbeg + 16 * t;
  const __nv_bfloat16* xb = x + (tok0 + g + 8 < M ? tok0 + g + 8 : M - 1) * (int64_t)D + kbeg + 16 * t;
  const __nv_bfloat16* wa = wq + (int64_t)g * D + kbeg + 16 * t;
  const __nv_bfloat16* wb = wq + (int64_t)(8 + g) * D + kbeg + 16 * t;
  float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
  for (int k0 = 0; k0 < dpart; k0 += 64) {
    uint32_t A0[8], A1[8], B0[8], B1[8];
    ld32B(xa + k0, A0);
    ld32B(xb + k0, A1);
    ld32B(wa + k0, B0);
    ld32B(wb + k0, B1);
#pragma unroll
    for (int st = 0; st < 4; ++st) {
      mma_bf16_16816(c0, A0[2 * st], A1[2 * st], A0[2 * st + 1], A1[2 * st + 1], B0[2 * st], B0[2 * st + 1]);
      mma_bf16_16816(c1, A0[2 * st], A1[2 * st], A0[2 * st + 1], A1[2 * st + 1], B1[2 * st], B1[2 * st + 1]);
    }
  }
  // c0: projections j = 2t, 2t+1 of rows g (c0[0..1]) and g+8 (c0[2..3]); c1: j = 8 + 2t, 9 + 2t
  float* q = sq + warp * 16 * 17;
  q[g * 17 + 2 * t] = c0[0];
  q[g * 17 + 2 * t + 1] = c0[1];
  q[(g + 8) * 17 + 2 * t] = c0[2];
  q[(g + 8) * 17 + 2 * t + 1] = c0[3];
  q[g * 17 + 8 + 2 * t] = c1[0];
  q[g * 17 + 9 + 2 * t] = c1[1];
  q[(g + 8) * 17 + 8 + 2 * t] = c1[2];
  q[(g + 8) * 17 + 9 + 2 * t] = c1[3];
  __syncthreads();
  const float eps = 1.1920928955078125e-07f;  // torch.finfo(float32).eps: F.rms_norm's default
  for (int r = warp * 4; r < warp * 4 + 4; ++r) {
    const int64_t tok = tok0 + r;
    if (tok >= M) break;
    float qv[16];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float v = sq[r * 17 + j];
#pragma unroll
      for (int w = 1; w < kMmaWarps; ++w) v += sq[w * 16 * 17 + r * 17 + j];
      qv[j] = v;
      ss = fmaf(v, v, ss);
    }
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(ss * (1.0f / 16.0f) + eps));
    float qown = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (lane == j) qown = qv[j];
      qv[j] *= inv;
    }
    if (q16_out && lane < 16) q16_out[tok * 16 + lane] = qown * inv;
    for (int b = lane; b < NB; b += 32) {
      float sc = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) sc = fmaf(qv[j], sk[j * NB + b], sc);
      scores[tok * NB + b] = sc * 0.25f;  // / sqrt(16)
    }
  }
}

// --------------------------------------------------------------------------------------------
// Selection: one warp per token row of scores.  Softmax over all blocks, base mass credit, stable
// descending order of remote probabilities (bitonic sort of 64-bit keys in per-warp shared memory),
// fp64-accumulated cumulative sum, count clamped to [K_min, min(available, K_max)].  Optionally the
// additive-stream context ctx16 = softmax(S/T) . K16.
// --------------------------------------------------------------------------------------------
constexpr int kSelWarps = 8;

__device__ __forceinline__ unsigned long long sel_key(float p, int b, bool remote) {
  // remote: (bits(p)+1, ~b) so that higher p first, then lower id; base: below every remote key.
  const uint32_t lo = 0xFFFFFFFFu - (uint32_t)b;
  return remote ? (((unsigned long long)(__float_as_uint(p) + 1u)) << 32) | lo : (unsigned long long)lo;
}

__device__ __forceinline__ unsigned long long shfl_xor_u64(unsigned long long v, int m) {
  const uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)v, m);
  const uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(v >> 32), m);
  return ((unsigned long long)hi << 32) | lo;
}

// Descending bitonic sort of N = 32*E keys held in registers, blocked layout: element i lives in
// lane i / E, register i % E.  Partners closer than E are in the same lane; farther ones are one
// shuffle away.  The network is fixed at compile time.
template <int E>
__device__ __forceinline__ void warp_bitonic_desc(unsigned long long (&v)[E], int lane) {
  constexpr int N = 32 * E;
#pragma unroll
  for (int k = 2; k <= N; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j < E) {
#pragma unroll
        for (int r = 0; r < E; ++r) {
          const int rp = r ^ j;
          if (rp > r) {
            const bool desc = (((lane * E + r) & k) == 0);
            const unsigned long long a = v[r], b = v[rp];
            const bool sw = desc ? (a < b) : (a > b);
            v[r] = sw ? b : a;
            v[rp] = sw ? a : b;
          }
        }
      } else {
        const int m = j / E;
        const bool lower = (lane & m) == 0;
#pragma unroll
        for (int r = 0; r < E; ++r) {
          const bool desc = (((lane * E + r) & k) == 0);
          const unsigned long long o = shfl_xor_u64(v[r], m);
          const bool keep_max = (desc == lower);
          v[r] = keep_max ? (v[r] > o ? v[r] : o) : (v[r] < o ? v[r] : o);
        }
      }
    }
  }
}

// One warp per token row of scores.  Softmax over all blocks (core.py:36-43), base mass credit
// (:104), stable descending order of remote probabilities (:105-108; ties -> lower id), fp64-accumulated
// cumulative sum (:109), count clamp (:111-119), sorted ids (:121-123).  Optionally the additive-stream
// context ctx16 = softmax(S/T) . K16 (foveal_pattention.py:339-340).
template <int E>
__global__ void __launch_bounds__(kSelWarps * 32)
select_blocks_kernel(const float* __restrict__ scores, int64_t M, int NB, int base, float top_p, int k_min,
                     int k_max, int capacity, float temperature, int32_t* __restrict__ out_idx,
                     int32_t* __restrict__ out_cnt, const float* __restrict__ k16f,
                     float* __restrict__ ctx16, float* __restrict__ stats, uint4* __restrict__ hzero,
                     int64_t hrow_vec) {
  constexpr int N = 32 * E;
  __shared__ float spb[kSelWarps][N];
  extern __shared__ float sk16[];  // [NB][16] fp32 block keys (only when ctx16 is requested)
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (ctx16) {
    for (int i = threadIdx.x; i < NB * 16; i += blockDim.x) sk16[i] = k16f[i];
    __syncthreads();
  }
  float* pbuf = spb[warp];
  for (int64_t tok = (int64_t)blockIdx.x * kSelWarps + warp; tok < M; tok += (int64_t)gridDim.x * kSelWarps) {
  const float* srow = scores + tok * NB;
  if (hzero) {  // clear this token's row of the masked activations H while the warp computes
    uint4* hr = hzero + tok * hrow_vec;
    for (int64_t i = lane; i < hrow_vec; i += 32) hr[i] = make_uint4(0u, 0u, 0u, 0u);
  }

  // blocked layout: lane owns blocks lane*E .. lane*E+E-1
  float p[E];
  float mx = -INFINITY;
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const int b = lane * E + r;
    float sv = -INFINITY;
    if (b < NB) {
      sv = srow[b];
      if (temperature != 1.0f) sv = __fdiv_rn(sv, temperature);
    }
    p[r] = sv;
    mx = fmaxf(mx, sv);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (!isfinite(mx)) mx = 0.f;
  float sum = 0.f;
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const int b = lane * E + r;
    const float e = b < NB ? expf(p[r] - mx) : 0.f;
    p[r] = e;
    sum += e;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float denom = fmaxf(sum, 1e-20f);
  unsigned long long key[E];
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const int b = lane * E + r;
    p[r] = __fdiv_rn(p[r], denom);
    key[r] = b < NB ? sel_key(p[r], b, b >= base) : 0ull;
    pbuf[b] = p[r];
  }
  __syncwarp();

  if (ctx16) {
    // lane L accumulates channel j = L % 16 over blocks b = L / 16, L / 16 + 2, ...: each load step reads
    // two contiguous 64-byte key rows; the two halves are combined with one shuffle
    const int j = lane & 15;
    float c = 0.f;
    for (int b = lane >> 4; b < NB; b += 2) c = fmaf(pbuf[b], sk16[b * 16 + j], c);
    c += __shfl_xor_sync(0xffffffffu, c, 16);
    if (lane < 16) ctx16[tok * 16 + j] = c;
  }
  if (out_idx == nullptr) { __syncwarp(); continue; }  // context-only mode

  // base (local) mass (core.py:104): sequential over the base blocks
  float local_mass = 0.f;
  if (lane == 0)
    for (int b = 0; b < base && b < NB; ++b) local_mass += pbuf[b];

  warp_bitonic_desc<E>(key, lane);

  int32_t* orow = out_idx + tok * capacity;
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const int i = lane * E + r;
    if (i < capacity) orow[i] = i < NB ? (int32_t)(0xFFFFFFFFu - (uint32_t)(key[r] & 0xFFFFFFFFull)) : 0;
    const uint32_t hi = (uint32_t)(key[r] >> 32);
    pbuf[i] = hi ? __uint_as_float(hi - 1u) : 0.f;  // sorted, clamped probabilities
  }
  for (int i = N + lane; i < capacity; i += 32) orow[i] = 0;
  __syncwarp();

  if (lane == 0) {
    float target = top_p - local_mass;
    target = target > 0.f ? target : 0.f;
    const int available = NB - base;
    int counts = 0;
    if (available > 0) {
      const int X = available < k_max ? available : k_max;
      int needed;
      if (target > 0.f) {
        double acc = 0.0;
        int n = 0;
        for (; n < X; ++n) {
          acc += (double)pbuf[n];
          if ((float)acc >= target) break;
        }
        needed = n + 1;  // #(cum < target) + 1; saturates at X + 1 when never reached within X
      } else {
        needed = 0;
      }
      needed = needed > k_min ? needed : k_min;
      counts = needed < available ? needed : available;
      counts = counts < k_max ? counts : k_max;
      if (counts < 0) counts = 0;
    }
    out_cnt[tok] = counts;
    if (stats) {
      atomicAdd(&stats[0], (k_max > 0 && counts >= k_max) ? 1.f : 0.f);
      atomicAdd(&stats[1], (float)counts);
      atomicAdd(&stats[2], counts == 0 ? 1.f : 0.f);
    }
  }
  __syncwarp();  // pbuf is rewritten by the next token of this warp
  }
}

// --------------------------------------------------------------------------------------------
// Block CSR (block-major token lists) in token chunks: key = chunk(t) * NBL + slot(b), where only
// blocks with b % stride == offset are local and slot(b) = b / stride.
// --------------------------------------------------------------------------------------------
__device__ __forceinline__ int token_block(int s, int base, const int32_t* ridx, int cap, int cnt) {
  // slot s < base: base block s; otherwise the (s-base)-th selected remote block, or -1
  if (s < base) return s;
  const int r = s - base;
  return r < cnt ? ridx[r] : -1;
}

// One CTA per kCsrTokens consecutive tokens (all inside one token chunk): block counts are gathered in
// a shared-memory histogram and folded into the global counts with one atomic per touched key.
constexpr int kCsrTokens = 128;

__global__ void __launch_bounds__(256)
csr_count_kernel(const int32_t* __restrict__ ridx, const int32_t* __restrict__ rcnt, int64_t M, int base,
                 int cap, int stride, int offset, int nbl, int chunk, int32_t* __restrict__ key_cnt) {
  extern __shared__ int32_t hist[];  // [nbl]
  for (int i = threadIdx.x; i < nbl; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int64_t t0 = (int64_t)blockIdx.x * kCsrTokens;
  const int slots = base + cap;
  const int64_t t_end = min(M, t0 + kCsrTokens);
  for (int64_t i = (int64_t)threadIdx.x; i < (t_end - t0) * slots; i += blockDim.x) {
    const int64_t t = t0 + i / slots;
    const int b = token_block((int)(i % slots), base, ridx + t * cap, cap, rcnt[t]);
    if (b >= 0 && (b % stride) == offset) atomicAdd(&hist[b / stride], 1);
  }
  __syncthreads();
  const int kbase = (int)(t0 / chunk) * nbl;
  for (int k = threadIdx.x; k < nbl; k += blockDim.x)
    if (hist[k]) atomicAdd(&key_cnt[kbase + k], hist[k]);
}

// Single CTA: exclusive scan of key counts and the tile list (key, first row); the tiles of one key
// have equal size (balanced_rows).
__global__ void __launch_bounds__(1024)
csr_scan_kernel(const int32_t* __restrict__ key_cnt, int nkey, int32_t* __restrict__ key_off,
                int32_t* __restrict__ key_fill, int2* __restrict__ tiles, int max_tiles,
                int32_t* __restrict__ meta, int* err) {
  __shared__ int s_pairs[1024], s_tiles[1024];
  const int tid = threadIdx.x;
  const int per = (nkey + 1023) / 1024;
  const int k0 = tid * per, k1 = min(nkey, k0 + per);
  int pairs = 0, ntile = 0;
  for (int k = k0; k < k1; ++k) {
    pairs += key_cnt[k];
    ntile += (key_cnt[k] + kGuN - 1) / kGuN;
  }
  s_pairs[tid] = pairs;
  s_tiles[tid] = ntile;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {  // Hillis-Steele inclusive scan
    const int a = tid >= o ? s_pairs[tid - o] : 0;
    const int b = tid >= o ? s_tiles[tid - o] : 0;
    __syncthreads();
    s_pairs[tid] += a;
    s_tiles[tid] += b;
    __syncthreads();
  }
  int poff = s_pairs[tid] - pairs, toff = s_tiles[tid] - ntile;
  for (int k = k0; k < k1; ++k) {
    const int c = key_cnt[k];
    key_off[k] = poff;
    key_fill[k] = 0;
    const int rows = balanced_rows(c);
    for (int r = 0; r < c; r += rows) {
      if (toff < max_tiles) tiles[toff] = make_int2(k, r);
      ++toff;
    }
    poff += c;
  }
  if (tid == 1023) {
    key_off[nkey] = s_pairs[1023];
    const int nt = s_tiles[1023];
    meta[0] = nt < max_tiles ? nt : max_tiles;
    meta[1] = s_pairs[1023];
    if (nt > max_tiles) record_error(err, kErrBadTile);
  }
}

// Same partition as csr_count_kernel: local histogram, one global reservation per key, then the
// scatter of token ids with shared-memory positions.
__global__ void __launch_bounds__(256)
csr_fill_kernel(const int32_t* __restrict__ ridx, const int32_t* __restrict__ rcnt, int64_t M, int base,
                int cap, int stride, int offset, int nbl, int chunk, const int32_t* __restrict__ key_off,
                int32_t* __restrict__ key_fill, int32_t* __restrict__ pair_tok) {
  extern __shared__ int32_t sh[];  // hist[nbl], start[nbl]
  int32_t* hist = sh;
  int32_t* start = sh + nbl;
  for (int i = threadIdx.x; i < nbl; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int64_t t0 = (int64_t)blockIdx.x * kCsrTokens;
  const int slots = base + cap;
  const int64_t t_end = min(M, t0 + kCsrTokens);
  const int64_t n = (t_end - t0) * slots;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const int64_t t = t0 + i / slots;
    const int b = token_block((int)(i % slots), base, ridx + t * cap, cap, rcnt[t]);
    if (b >= 0 && (b % stride) == offset) atomicAdd(&hist[b / stride], 1);
  }
  __syncthreads();
  const int kbase = (int)(t0 / chunk) * nbl;
  for (int k = threadIdx.x; k < nbl; k += blockDim.x) {
    start[k] = hist[k] ? key_off[kbase + k] + atomicAdd(&key_fill[kbase + k], hist[k]) : 0;
    hist[k] = 0;
  }
  __syncthreads();
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const int64_t t = t0 + i / slots;
    const int b = token_block((int)(i % slots), base, ridx + t * cap, cap, rcnt[t]);
    if (b >= 0 && (b % stride) == offset) {
      const int k = b / stride;
      pair_tok[start[k] + atomicAdd(&hist[k], 1)] = (int32_t)t;
    }
  }
}

// --------------------------------------------------------------------------------------------
// Pooled routing.
// --------------------------------------------------------------------------------------------
constexpr int kColRows = 256;

// partial column sums over kColRows-row chunks: part[chunk][d]
template <typename T>
__global__ void colsum_partial_kernel(const T* __restrict__ a, int64_t M, int D, float* __restrict__ part) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= D) return;
  const int64_t r0 = (int64_t)blockIdx.y * kColRows;
  const int64_t r1 = min(M, r0 + kColRows);
  float s = 0.f;
  for (int64_t r = r0; r < r1; ++r) s += to_f32(a[r * D + d]);
  part[(int64_t)blockIdx.y * D + d] = s;
}
__global__ void colsum_final_kernel(const float* __restrict__ part, int nchunk, int64_t M, int D,
                                    float* __restrict__ mean) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= D) return;
  float s = 0.f;
  for (int c = 0; c < nchunk; ++c) s += part[(int64_t)c * D + d];
  mean[d] = __fdiv_rn(s, (float)M);
}

__device__ __forceinline__ uint32_t orderable(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Single CTA of 512 threads.  mode 0 (eval): mean_vec is the token-mean of x [D]; the pooled query
// q = rms_norm(W_q mean), scores = q . K16^T (no 1/sqrt(16), foveal_pattention.py:312-313).
// mode 1 (train): mean_vec is the token-mean of the per-token scores [NB].  Then top-k over the
// remote blocks, ordered by descending score (ties: lower id), base ids first.
template <typename T>
__global__ void __launch_bounds__(512)
pooled_topk_kernel(const float* __restrict__ mean_vec, const T* __restrict__ wq, const T* __restrict__ k16,
                   int D, int NB, int nb_pad, int base, int remote, int mode, int32_t* __restrict__ active,
                   float* __restrict__ mean_scores_out) {
  extern __shared__ unsigned long long pk[];  // [nb_pad]
  __shared__ float sq[16];
  __shared__ float sscore[4096];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (mode == 0) {
    if (warp < 16) {
      float acc = 0.f;
      for (int d = lane; d < D; d += 32) acc = fmaf(mean_vec[d], to_f32(wq[(int64_t)warp * D + d]), acc);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) sq[warp] = acc;
    }
    __syncthreads();
    if (tid == 0) {
      float ss = 0.f;
      for (int j = 0; j < 16; ++j) ss = fmaf(sq[j], sq[j], ss);
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(ss * (1.0f / 16.0f) + 1.1920928955078125e-07f));
      for (int j = 0; j < 16; ++j) sq[j] = sq[j] * inv;
    }
    __syncthreads();
    for (int b = tid; b < NB; b += blockDim.x) {
      float s = 0.f;
      for (int j = 0; j < 16; ++j) s = fmaf(sq[j], to_f32(k16[b * 16 + j]), s);
      sscore[b] = s;
    }
  } else {
    for (int b = tid; b < NB; b += blockDim.x) sscore[b] = mean_vec[b];
  }
  __syncthreads();
  for (int b = tid; b < nb_pad; b += blockDim.x) {
    unsigned long long key = 0ull;
    if (b < NB && b >= base)
      key = ((unsigned long long)orderable(sscore[b]) << 32) | (0xFFFFFFFFu - (uint32_t)b);
    pk[b] = key;
    if (mean_scores_out && b < NB) mean_scores_out[b] = sscore[b];
  }
  __syncthreads();
  for (int k = 2; k <= nb_pad; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int idx = tid; idx < (nb_pad >> 1); idx += blockDim.x) {
        const int i = 2 * j * (idx / j) + (idx % j);
        const int l = i + j;
        const unsigned long long a = pk[i], bb = pk[l];
        const bool desc = (i & k) == 0;
        if (desc ? (a < bb) : (a > bb)) { pk[i] = bb; pk[l] = a; }
      }
      __syncthreads();
    }
  }
  for (int i = tid; i < base + remote; i += blockDim.x) {
    active[i] = i < base ? i : (int32_t)(0xFFFFFFFFu - (uint32_t)(pk[i - base] & 0xFFFFFFFFull));
  }
}

// ============================================================================================
// Host launchers
// ============================================================================================
int launch_router_scores(const void* x, const void* wq, const void* k16, int dtype, int64_t M, int D,
                         int NB, float temperature, float* scores, float* q16, cudaStream_t st) {
  if (M <= 0) return FP_OK;
  if (dtype == FP_DTYPE_BF16 && D % (64 * kMmaWarps) == 0 && temperature == 1.0f) {
    const size_t smem = (size_t)NB * 16 * sizeof(float) + kMmaWarps * 16 * 17 * sizeof(float);
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(router_scores_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
      return FP_ERR_CUDA;
    const int blocks = (int)((M + 15) / 16);
    router_scores_mma_kernel<<<blocks, kMmaWarps * 32, smem, st>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)wq, (const __nv_bfloat16*)k16, M, D, NB, scores, q16);
    return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
  }
  const int blocks = (int)((M + kScoreWarps * kScoreTPW - 1) / (kScoreWarps * kScoreTPW));
  const size_t smem = (size_t)NB * 16 * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = dtype == FP_DTYPE_BF16
        ? cudaFuncSetAttribute(router_scores_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)
        : cudaFuncSetAttribute(router_scores_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return FP_ERR_CUDA;
  }
  if (dtype == FP_DTYPE_BF16)
    router_scores_kernel<__nv_bfloat16><<<blocks, kScoreWarps * 32, smem, st>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)wq, (const __nv_bfloat16*)k16, M, D, NB, 0.25f,
        temperature, scores, q16);
  else
    router_scores_kernel<float><<<blocks, kScoreWarps * 32, smem, st>>>(
        (const float*)x, (const float*)wq, (const float*)k16, M, D, NB, 0.25f, temperature, scores, q16);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

static int pow2_at_least(int n) {
  int p = 32;
  while (p < n) p <<= 1;
  return p;
}

__global__ void convert_keys_kernel(const void* k16, int dtype, int n, float* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  out[i] = dtype == FP_DTYPE_BF16 ? __bfloat162float(((const __nv_bfloat16*)k16)[i]) : ((const float*)k16)[i];
}

int launch_select(const float* scores, int64_t M, int NB, int base, float top_p, int k_min, int k_max,
                  int capacity, float temperature, int32_t* idx, int32_t* cnt, const float* k16f,
                  float* ctx16, float* stats, cudaStream_t st, void* hzero, int64_t hrow_bytes) {
  if (M <= 0) return FP_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t need = (M + kSelWarps - 1) / kSelWarps;
  const int blocks = (int)std::min<int64_t>(need, (int64_t)sms * 8);
  const size_t smem = ctx16 ? (size_t)NB * 16 * sizeof(float) : 0;
  auto go = [&](auto kern) {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return FP_ERR_CUDA;
    kern<<<blocks, kSelWarps * 32, smem, st>>>(scores, M, NB, base, top_p, k_min, k_max, capacity, temperature,
                                               idx, cnt, k16f, ctx16, stats, (uint4*)hzero, hrow_bytes / 16);
    return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
  };
  if (NB <= 32) return go(select_blocks_kernel<1>);
  if (NB <= 64) return go(select_blocks_kernel<2>);
  if (NB <= 128) return go(select_blocks_kernel<4>);
  if (NB <= 256) return go(select_blocks_kernel<8>);
  if (NB <= 512) return go(select_blocks_kernel<16>);
  if (NB <= 1024) return go(select_blocks_kernel<32>);
  return FP_ERR_UNSUPPORTED;
}

int launch_convert_keys(const void* k16, int dtype, int n, float* out, cudaStream_t st) {
  convert_keys_kernel<<<(n + 255) / 256, 256, 0, st>>>(k16, dtype, n, out);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

int launch_build_csr(const int32_t* ridx, const int32_t* rcnt, int64_t M, int base, int cap, int stride,
                     int offset, int nbl, int chunk, int nkey, int32_t* key_cnt, int32_t* key_off,
                     int32_t* key_fill, int32_t* pair_tok, int2* tiles, int max_tiles, int32_t* meta, int* err,
                     cudaStream_t st) {
  if (chunk % kCsrTokens) return FP_ERR_INVALID_ARG;
  if (cudaMemsetAsync(key_cnt, 0, sizeof(int32_t) * nkey, st) != cudaSuccess) return FP_ERR_CUDA;
  const int blocks = (int)((M + kCsrTokens - 1) / kCsrTokens);
  if (blocks > 0)
    csr_count_kernel<<<blocks, 256, nbl * sizeof(int32_t), st>>>(ridx, rcnt, M, base, cap, stride, offset, nbl,
                                                                chunk, key_cnt);
  csr_scan_kernel<<<1, 1024, 0, st>>>(key_cnt, nkey, key_off, key_fill, tiles, max_tiles, meta, err);
  if (blocks > 0)
    csr_fill_kernel<<<blocks, 256, 2 * nbl * sizeof(int32_t), st>>>(ridx, rcnt, M, base, cap, stride, offset, nbl,
                                                                    chunk, key_off, key_fill, pair_tok);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

int launch_colmean(const void* a, int dtype, int64_t M, int D, float* part, float* mean, cudaStream_t st) {
  const int nchunk = (int)((M + kColRows - 1) / kColRows);
  dim3 g((D + 255) / 256, nchunk);
  if (dtype == FP_DTYPE_BF16)
    colsum_partial_kernel<__nv_bfloat16><<<g, 256, 0, st>>>((const __nv_bfloat16*)a, M, D, part);
  else
    colsum_partial_kernel<float><<<g, 256, 0, st>>>((const float*)a, M, D, part);
  colsum_final_kernel<<<(D + 255) / 256, 256, 0, st>>>(part, nchunk, M, D, mean);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

int launch_pooled_topk(const float* mean_vec, const void* wq, const void* k16, int dtype, int D, int NB,
                       int base, int remote, int mode, int32_t* active, float* mean_scores_out,
                       cudaStream_t st) {
  const int nb_pad = pow2_at_least(NB);
  const size_t smem = (size_t)nb_pad * sizeof(unsigned long long);
  if (dtype == FP_DTYPE_BF16)
    pooled_topk_kernel<__nv_bfloat16><<<1, 512, smem, st>>>(mean_vec, (const __nv_bfloat16*)wq,
                                                            (const __nv_bfloat16*)k16, D, NB, nb_pad, base,
                                                            remote, mode, active, mean_scores_out);
  else
    pooled_topk_kernel<float><<<1, 512, smem, st>>>(mean_vec, (const float*)wq, (const float*)k16, D, NB,
                                                    nb_pad, base, remote, mode, active, mean_scores_out);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

}  // namespace fp
