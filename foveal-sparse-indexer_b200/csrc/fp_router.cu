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
#include <type_traits>
#include <mutex>

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
                     float* __restrict__ scores, float* __restrict__ q16_out, const float* __restrict__ kcos) {
  extern __shared__ float sk[];  // [16][NB] fp32 block keys, transposed: lanes read consecutive blocks
  if (kcos) {
    // cosine form: keys L2-normalised in fp32 (F.normalize: k / max(||k||, 1e-12))
    for (int b = threadIdx.x; b < NB; b += blockDim.x) {
      float kv[16], ss = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        kv[j] = kcos[b * 16 + j];
        ss = fmaf(kv[j], kv[j], ss);
      }
      const float nrm = fmaxf(__fsqrt_rn(ss), 1e-12f);
#pragma unroll
      for (int j = 0; j < 16; ++j) sk[j * NB + b] = __fdiv_rn(kv[j], nrm);
    }
  } else {
    for (int i = threadIdx.x; i < NB * 16; i += blockDim.x) sk[(i & 15) * NB + (i >> 4)] = to_f32(k16[i]);
  }
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
    if (kcos) {  // normalize(rms_norm(q)) of compute_block_scores
      float qq = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) qq = fmaf(q[j], q[j], qq);
      const float nrm = fmaxf(__fsqrt_rn(qq), 1e-12f);
#pragma unroll
      for (int j = 0; j < 16; ++j) q[j] = __fdiv_rn(q[j], nrm);
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
                         float* __restrict__ scores, float* __restrict__ q16_out, const float* __restrict__ kcos) {
  extern __shared__ float sk[];  // [16][NB] transposed block keys, then [kMmaWarps][16][17] partials
  float* sq = sk + 16 * NB;
  if (kcos) {
    // cosine form: fp32 keys, L2-normalised (F.normalize: k / max(||k||, 1e-12))
    for (int b = threadIdx.x; b < NB; b += blockDim.x) {
      float kv[16], ss = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        kv[j] = kcos[b * 16 + j];
        ss = fmaf(kv[j], kv[j], ss);
      }
      const float nrm = fmaxf(__fsqrt_rn(ss), 1e-12f);
#pragma unroll
      for (int j = 0; j < 16; ++j) sk[j * NB + b] = __fdiv_rn(kv[j], nrm);
    }
  } else {
    for (int i = threadIdx.x; i < NB * 16; i += blockDim.x) sk[(i & 15) * NB + (i >> 4)] = __bfloat162float(k16[i]);
  }
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
    if (kcos) {  // normalize(rms_norm(q)) of compute_block_scores
      float qq = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) qq = fmaf(qv[j], qv[j], qq);
      const float nrm = fmaxf(__fsqrt_rn(qq), 1e-12f);
#pragma unroll
      for (int j = 0; j < 16; ++j) qv[j] = __fdiv_rn(qv[j], nrm);
    }
    for (int b = lane; b < NB; b += 32) {
      float sc = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) sc = fmaf(qv[j], sk[j * NB + b], sc);
      scores[tok * NB + b] = sc * 0.25f;  // / sqrt(16)
    }
  }
}

// --------------------------------------------------------------------------------------------
// Selection: one warp per token.  Softmax over all blocks, base mass credit, stable descending order
// of remote probabilities (bitonic sort of 64-bit keys in registers), fp64-accumulated cumulative
// sum, count clamped to [K_min, min(available, K_max)].  Optionally the additive-stream context
// ctx16 = softmax(S/T) . K16.
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

// Descending bitonic sort of N = 32*E keys held in registers.  The result is in blocked layout
// (element i in lane i / E, register i % E); the input arrangement is arbitrary.  Merge stages are
// runtime loops (small code: one warp sorts one token while its neighbours run the same few hundred
// instructions); only the register-local steps are unrolled.
template <int E>
__device__ __forceinline__ void warp_bitonic_desc(unsigned long long (&v)[E], int lane) {
  constexpr int N = 32 * E;
#pragma unroll 1
  for (int k = 2; k <= N; k <<= 1) {
#pragma unroll 1
    for (int j = k >> 1; j >= E; j >>= 1) {  // partner in lane ^ (j / E)
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
#pragma unroll
    for (int j = E >> 1; j > 0; j >>= 1) {  // partner in the same lane
      if (j < k) {
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
      }
    }
  }
}

// Top `need` keys in descending order without sorting all N: the need-th largest probability word T
// is found by a bitwise search with warp-wide counts (only the bits below the common prefix of the
// smallest and largest remote word are searched), the keys with hi word >= T are compacted into cbuf
// (C slots) and only those are sorted.  Result in blocked layout (position lane*(C/32) + q in out[q]).
// Returns false, with nothing sorted, when more than C keys tie at or above T.
template <int E, int C>
__device__ __forceinline__ bool sort_top(const unsigned long long (&key)[E], int need, unsigned long long* cbuf,
                                         unsigned long long (&out)[C / 32], int lane) {
  uint32_t hi[E];
  uint32_t mx = 0u, mn = 0xFFFFFFFFu;
#pragma unroll
  for (int r = 0; r < E; ++r) {
    hi[r] = (uint32_t)(key[r] >> 32);  // remote keys: bits(p) + 1 >= 1; base and padding: 0
    mx = hi[r] > mx ? hi[r] : mx;
    if (hi[r] != 0u && hi[r] < mn) mn = hi[r];
  }
  mx = __reduce_max_sync(0xffffffffu, mx);
  mn = __reduce_min_sync(0xffffffffu, mn);
  const uint32_t diff = mn ^ mx;
  int bit = diff ? 31 - __clz(diff) : -1;
  uint32_t T = diff ? (mx & ~((2u << bit) - 1u)) : mx;  // bits above `bit` are common to [mn, mx]
  for (; bit >= 0; --bit) {
    const uint32_t cand = T | (1u << bit);
    int c = 0;
#pragma unroll
    for (int r = 0; r < E; ++r) c += hi[r] >= cand ? 1 : 0;
    if (__reduce_add_sync(0xffffffffu, c) >= need) T = cand;
  }
  int total = 0;
  const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const bool f = hi[r] >= T;
    const uint32_t bal = __ballot_sync(0xffffffffu, f);
    const int pos = total + __popc(bal & lt);
    if (f && pos < C) cbuf[pos] = key[r];
    total += __popc(bal);
  }
  if (total > C) return false;
  __syncwarp();
#pragma unroll
  for (int q = 0; q < C / 32; ++q) {
    const int i = lane * (C / 32) + q;
    out[q] = i < total ? cbuf[i] : 0ull;
  }
  __syncwarp();  // cbuf may be rewritten from here on
  warp_bitonic_desc<C / 32>(out, lane);
  return true;
}

// Top `need` keys in descending order by `need` rounds of a warp-wide maximum (64-bit keys: the high words
// first, then the low words among the lanes holding the top high word), each round retiring the key it
// found from its lane.  Result in blocked layout (position lane * Q + q in out[q]; positions >= need: 0).
// For need <= 32 this is several times shorter than the threshold search + compaction + bitonic sort of
// sort_top (measured 4.0 us for need = 8 on one warp), and it returns the same keys in the same order.
template <int E, int Q>
__device__ __forceinline__ void top_by_rounds(const unsigned long long (&key)[E], int need,
                                              unsigned long long (&out)[Q], int lane) {
  unsigned long long k[E];
#pragma unroll
  for (int r = 0; r < E; ++r) k[r] = key[r];
#pragma unroll
  for (int q = 0; q < Q; ++q) out[q] = 0ull;
  for (int i = 0; i < need; ++i) {
    unsigned long long lm = 0ull;
#pragma unroll
    for (int r = 0; r < E; ++r) lm = k[r] > lm ? k[r] : lm;
    const uint32_t hi = (uint32_t)(lm >> 32);
    const uint32_t mhi = __reduce_max_sync(0xffffffffu, hi);
    const uint32_t mlo = __reduce_max_sync(0xffffffffu, hi == mhi ? (uint32_t)lm : 0u);
    const unsigned long long w = ((unsigned long long)mhi << 32) | mlo;
#pragma unroll
    for (int r = 0; r < E; ++r)
      if (k[r] == w) k[r] = 0ull;  // keys are distinct (the low word holds the block id)
#pragma unroll
    for (int q = 0; q < Q; ++q)
      if (i == lane * Q + q) out[q] = w;
  }
}

// Selection of one token on one warp.  s[r] is the (temperature-scaled) score of block r*32 + lane.
// pbuf: this warp's shared row of 32*E floats; sbuf (optional): shared row receiving the sorted block
// ids; skT (needed with ctx16): [16][ks] fp32 block keys, transposed (row stride ks >= NB).  Returns the
// remote count on every lane (0 in context-only mode).
// Reference: masked_softmax core.py:36-43; select_blocks core.py:101-123 (base mass :104, stable
// descending order :105-108 with ties to the lower id, cumsum :109, clamp :111-119, ids :121-123);
// context foveal_pattention.py:339-340.
template <int E>
__device__ __forceinline__ int select_token(float (&s)[E], int64_t tok, const SelectOut& o, float* pbuf,
                                            int32_t* sbuf, const float* skT, int ks, int lane) {
  constexpr int N = 32 * E;
  const int NB = o.NB;
  float mx = -INFINITY;
#pragma unroll
  for (int r = 0; r < E; ++r) {
    if (r * 32 + lane >= NB) s[r] = -INFINITY;
    mx = fmaxf(mx, s[r]);
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
  if (!isfinite(mx)) mx = 0.f;
  float sum = 0.f;
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const float e = r * 32 + lane < NB ? expf(s[r] - mx) : 0.f;
    s[r] = e;
    sum += e;
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, m);
  const float denom = fmaxf(sum, 1e-20f);
  unsigned long long key[E];
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const int b = r * 32 + lane;
    s[r] = __fdiv_rn(s[r], denom);
    key[r] = b < NB ? sel_key(s[r], b, b >= o.base) : 0ull;
    pbuf[b] = s[r];
  }
  if (o.ctx16) {
    // lane-partial context over this lane's blocks, then a butterfly reduce-scatter: after the steps
    // over lane bits 4..1 lane L holds channel (L >> 1) summed over 16 lanes; the last step adds L ^ 1
    float c[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) c[j] = 0.f;
#pragma unroll
    for (int r = 0; r < E; ++r) {
      const int b = r * 32 + lane;
      if (b < NB) {
#pragma unroll
        for (int j = 0; j < 16; ++j) c[j] = fmaf(s[r], skT[j * ks + b], c[j]);
      }
    }
#pragma unroll
    for (int h = 8; h >= 1; h >>= 1) {  // 16 -> 8 -> 4 -> 2 -> 1 values per lane
      const bool up = (lane & (2 * h)) != 0;
#pragma unroll
      for (int i = 0; i < h; ++i) {
        const float send = up ? c[i] : c[i + h];
        const float keep = up ? c[i + h] : c[i];
        c[i] = keep + __shfl_xor_sync(0xffffffffu, send, 2 * h);
      }
    }
    c[0] += __shfl_xor_sync(0xffffffffu, c[0], 1);
    if ((lane & 1) == 0) o.ctx16[tok * 16 + (lane >> 1)] = c[0];
  }
  if (o.idx == nullptr) return 0;  // context-only mode
  __syncwarp();

  // base (local) mass (core.py:104): sequential over the base blocks
  float local_mass = 0.f;
  if (lane == 0)
    for (int b = 0; b < o.base && b < NB; ++b) local_mass += pbuf[b];
  __syncwarp();

  const int avail = NB - o.base;
  const int X = avail < o.k_max ? avail : o.k_max;  // positions the cumulative sum may need
  const int need = o.capacity > X ? o.capacity : X;  // sorted positions required
  int32_t* orow = o.idx + tok * o.capacity;
  bool done = false;
  auto emit = [&](unsigned long long kv, int i) {
    const int32_t id = i < NB ? (int32_t)(0xFFFFFFFFu - (uint32_t)(kv & 0xFFFFFFFFull)) + o.id_offset : 0;
    if (i < o.capacity) orow[i] = id;
    if (sbuf) sbuf[i] = id;
    const uint32_t hi = (uint32_t)(kv >> 32);
    pbuf[i] = hi ? __uint_as_float(hi - 1u) : 0.f;  // sorted, clamped probabilities
  };
  float target = o.top_p - local_mass;  // lane 0's local mass; broadcast below
  target = __shfl_sync(0xffffffffu, target, 0);
  target = target > 0.f ? target : 0.f;
  int below = -1;  // #(cum < target) among the first X sorted probabilities, when found in registers
  // Cumulative sum of the sorted probabilities held in registers (Q consecutive positions per lane).
  // The reference accumulates sequentially in fp64 and rounds each prefix to fp32.  When every summand
  // is 0 or >= 2^-29, all partial sums are multiples of 2^-52 below 2, so fp64 addition is exact and
  // a warp scan gives the same prefixes; otherwise the sequential loop below runs.
  auto scan_count = [&](const auto& top, auto qconst) {
    constexpr int Q = decltype(qconst)::value;
    float pv[Q];
    bool ok = true;
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const uint32_t hi = (uint32_t)(top[q] >> 32);
      pv[q] = (lane * Q + q < X && hi) ? __uint_as_float(hi - 1u) : 0.f;
      ok = ok && (pv[q] == 0.f || pv[q] >= 0x1p-29f);
    }
    if (!__all_sync(0xffffffffu, ok)) return;
    double own = 0.0;
#pragma unroll
    for (int q = 0; q < Q; ++q) own += (double)pv[q];
    double incl = own;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
      const double up = __shfl_up_sync(0xffffffffu, incl, m);
      if (lane >= m) incl += up;
    }
    double c = incl - own;  // exact (all values are multiples of 2^-52 below 2)
    int n = 0;
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      c += (double)pv[q];
      n += __popc(__ballot_sync(0xffffffffu, lane * Q + q < X && (float)c < target));
    }
    below = n;
  };
  {
    // Q positions per lane, so that every emitted position stays inside this warp's 32 * E slots of
    // pbuf / sbuf (E = 1: 32 positions)
    constexpr int Q = E >= 2 ? 2 : 1;
    if (need >= 1 && need <= 32 && need <= 32 * Q && avail >= need) {
      unsigned long long top[Q];
      top_by_rounds<E, Q>(key, need, top, lane);
#pragma unroll
      for (int q = 0; q < Q; ++q) emit(top[q], Q * lane + q);
      if (target > 0.f) scan_count(top, std::integral_constant<int, Q>{});
      done = true;
    }
  }
  if constexpr (E >= 4) {
    if (!done && need >= 1 && need <= 64 && avail >= need) {
      unsigned long long top[2];
      if (sort_top<E, 64>(key, need, reinterpret_cast<unsigned long long*>(pbuf), top, lane)) {
        emit(top[0], 2 * lane);
        emit(top[1], 2 * lane + 1);
        if (target > 0.f) scan_count(top, std::integral_constant<int, 2>{});
        done = true;
      }
    }
  }
  if constexpr (E >= 8) {
    if (!done && need > 64 && need <= 128 && avail >= need) {
      unsigned long long top[4];
      if (sort_top<E, 128>(key, need, reinterpret_cast<unsigned long long*>(pbuf), top, lane)) {
#pragma unroll
        for (int q = 0; q < 4; ++q) emit(top[q], 4 * lane + q);
        if (target > 0.f) scan_count(top, std::integral_constant<int, 4>{});
        done = true;
      }
    }
  }
  if (!done) {  // full sort of all N keys
    warp_bitonic_desc<E>(key, lane);
#pragma unroll
    for (int r = 0; r < E; ++r) emit(key[r], lane * E + r);
    for (int i = N + lane; i < o.capacity; i += 32) orow[i] = 0;
  }
  __syncwarp();

  int counts = 0;
  if (lane == 0) {
    if (avail > 0) {
      int needed = 0;
      if (target > 0.f) {
        if (below < 0) {
          // sequential fp64 cumulative sum over the first X sorted probabilities (the prefix is
          // monotone, so counting prefixes below the target equals the reference's count once clamped)
          double acc = 0.0;
          below = 0;
          for (int q = 0; q < X; q += 4) {
            const float4 v4 = *reinterpret_cast<const float4*>(pbuf + q);
            const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              if (q + u < X) {
                acc += (double)vv[u];
                below += (float)acc < target ? 1 : 0;
              }
            }
          }
        }
        needed = below + 1;
      } else if (o.fast) {
        needed = 1;
      }
      needed = needed > o.k_min ? needed : o.k_min;
      counts = (o.fast || needed < avail) ? needed : avail;
      counts = counts < o.k_max ? counts : o.k_max;
      if (counts < 0) counts = 0;
    }
    o.cnt[tok] = counts;
  }
  counts = __shfl_sync(0xffffffffu, counts, 0);
  return counts;
}

// Standalone selection over a score matrix (fp_select_blocks): one warp per token row, persistent.
template <int E>
__global__ void __launch_bounds__(kSelWarps * 32)
select_blocks_kernel(const float* __restrict__ scores, int64_t M, float temperature, const SelectOut o,
                     const float* __restrict__ k16f) {
  constexpr int N = 32 * E;
  extern __shared__ float4 sel_smem4[];
  float* pball = reinterpret_cast<float*>(sel_smem4);  // [kSelWarps][N]
  float* skT = pball + kSelWarps * N;                  // [16][NB] (only with ctx16)
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (o.ctx16) {
    for (int i = threadIdx.x; i < o.NB * 16; i += blockDim.x) {
      const int j = i / o.NB, b = i - j * o.NB;
      skT[i] = k16f[b * 16 + j];
    }
    __syncthreads();
  }
  float* pbuf = pball + warp * N;
  // statistics (capped tokens, sum of counts, base-only tokens): integers, summed per warp in registers,
  // then per CTA, with one atomic per CTA and statistic
  int st_cap = 0, st_zero = 0;
  long long st_sum = 0;
  for (int64_t tok = (int64_t)blockIdx.x * kSelWarps + warp; tok < M; tok += (int64_t)gridDim.x * kSelWarps) {
    const float* srow = scores + tok * (o.ld > 0 ? o.ld : (int64_t)o.NB);
    float s[E];
#pragma unroll
    for (int r = 0; r < E; ++r) {
      const int b = r * 32 + lane;
      float v = -INFINITY;
      if (b < o.NB) {
        v = srow[b];
        if (temperature != 1.0f) v = __fdiv_rn(v, temperature);
      }
      s[r] = v;
    }
    const int c = select_token<E>(s, tok, o, pbuf, nullptr, skT, o.NB, lane);
    st_cap += (o.k_max > 0 && c >= o.k_max) ? 1 : 0;
    st_sum += c;
    st_zero += c == 0 ? 1 : 0;
    __syncwarp();  // pbuf is rewritten by the next token of this warp
  }
  if (o.stats && o.idx) {
    __shared__ long long red[kSelWarps][3];
    if (lane == 0) {
      red[warp][0] = st_cap;
      red[warp][1] = st_sum;
      red[warp][2] = st_zero;
    }
    __syncthreads();
    if (threadIdx.x < 3) {
      long long t = 0;
      for (int w = 0; w < kSelWarps; ++w) t += red[w][threadIdx.x];
      if (t) atomicAdd(&o.stats[threadIdx.x], (float)t);
    }
  }
}

// --------------------------------------------------------------------------------------------
// Fused token routing of the forward: scores, selection and the block-major token lists in one
// kernel.  A CTA routes 16 tokens: its warps first split the 16-D projection x W_q^T over the hidden
// dimension (mma.sync bf16, or fp32 FFMA with one warp per token), then each warp finishes its
// token(s): RMSNorm, the NB block scores, the selection, and the block-CSR entries.
//
// Block CSR: key = chunk(t) * NBL + slot(b) (token chunks of `chunk` tokens; only blocks with
// b % stride == offset are local, slot(b) = b / stride).  Every key owns a fixed bucket of key_cap
// entries of pair_tok (a token enters a key at most once), filled through an atomic counter per key,
// so no separate counting pass is needed; the order of tokens inside a bucket does not change any
// result (each token column of a gate/up tile is computed independently).  The last CTA to finish
// (atomic ticket) turns the key counts into the gate/up tile list.
// --------------------------------------------------------------------------------------------
// Raises a kernel's dynamic shared-memory limit once per kernel (to the largest size asked so far).
template <auto Kern>
int ensure_smem(size_t smem) {
  static std::mutex mu;
  static size_t granted = 48 * 1024;
  if (smem <= 48 * 1024) return FP_OK;
  std::lock_guard<std::mutex> lock(mu);
  if (smem <= granted) return FP_OK;
  if (cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return FP_ERR_CUDA;
  granted = smem;
  return FP_OK;
}

constexpr int kRouteWarps = 8;
constexpr int kProjTokens = 16;                           // tokens per projection CTA (the mma.sync M dimension)
constexpr int kProjTPW = kProjTokens / kRouteWarps;       // tokens per warp of the projection's FFMA form
constexpr int kRouteTPW = 1;                              // tokens per warp in a routing group
constexpr int kRouteTokens = kRouteWarps * kRouteTPW;     // tokens per routing group (at most 16)
static_assert(kRouteTokens <= 16, "group-local pair positions are packed in 4 bits");
constexpr uint32_t kRouteZeroBytes = 16384;               // zero source of the bulk H clears

// Dynamic shared-memory layout of route_kernel (byte offsets, 16-byte aligned).
struct RouteSmem {
  int zbuf, skT, pbuf, sbuf, plist, cnt, kbase, total;
};
__host__ __device__ inline RouteSmem route_smem(int NB, int nbl, int E, bool hz, bool csr) {
  auto al = [](int v) { return (v + 15) & ~15; };
  const int N = 32 * E, nbp = (NB + 3) & ~3;
  RouteSmem L;
  int o = 0;
  L.zbuf = o;  o += hz ? (int)kRouteZeroBytes : 0;
  L.skT = o;   o += al(16 * nbp * 4);
  L.pbuf = o;  o += kRouteWarps * N * 4;
  L.sbuf = o;  o += kRouteWarps * N * 4;
  L.plist = o; o += csr ? kRouteTokens * N * 4 : 0;
  L.cnt = o;   o += csr ? al(nbl * 4) : 0;
  L.kbase = o; o += csr ? al(nbl * 4) : 0;
  L.total = o;
  return L;
}

// Gate/up tile list from the key counts (one CTA): exclusive scan of per-key tile counts, then the
// (key, first row) descriptor of every tile in key order.
__device__ void build_tile_list(const RouteArgs& a) {
  __shared__ int s_wp[32], s_wt[32];
  const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, warp = tid >> 5;
  const int per = (a.nkey + nth - 1) / nth;
  const int k0 = min(a.nkey, tid * per), k1 = min(a.nkey, k0 + per);
  int pairs = 0, ntile = 0;
  for (int k = k0; k < k1; ++k) {
    const int c = __ldcg(&a.key_cnt[k]);
    pairs += c;
    ntile += (c + kGuN - 1) / kGuN;
  }
  int ip = pairs, it = ntile;  // inclusive warp scan
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const int up = __shfl_up_sync(0xffffffffu, ip, m), ut = __shfl_up_sync(0xffffffffu, it, m);
    if (lane >= m) { ip += up; it += ut; }
  }
  if (lane == 31) { s_wp[warp] = ip; s_wt[warp] = it; }
  __syncthreads();
  if (warp == 0) {
    const int nw = nth >> 5;
    int wp = lane < nw ? s_wp[lane] : 0, wt = lane < nw ? s_wt[lane] : 0;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
      const int up = __shfl_up_sync(0xffffffffu, wp, m), ut = __shfl_up_sync(0xffffffffu, wt, m);
      if (lane >= m) { wp += up; wt += ut; }
    }
    if (lane < nw) { s_wp[lane] = wp; s_wt[lane] = wt; }  // inclusive over warps
  }
  __syncthreads();
  int toff = (warp > 0 ? s_wt[warp - 1] : 0) + it - ntile;
  for (int k = k0; k < k1; ++k) {
    const int c = __ldcg(&a.key_cnt[k]);
    const int rows = balanced_rows(c);
    for (int r = 0; r < c; r += rows) {
      if (toff < a.max_tiles) a.tiles[toff] = make_int2(k, r);
      ++toff;
    }
  }
  if (tid == nth - 1) {
    const int nw = nth >> 5;
    const int nt = s_wt[nw - 1];
    a.meta[0] = nt < a.max_tiles ? nt : a.max_tiles;
    a.meta[1] = s_wp[nw - 1];
    if (nt > a.max_tiles) record_error(a.err, kErrBadTile);
  }
}

// Stage the block keys K16 [NB][16] transposed into skT[16][nbp] (fp32).  One thread per key row:
// vector loads when the rows are 16-byte aligned.
template <typename T>
__device__ __forceinline__ void stage_keys(const T* __restrict__ k16, int NB, int nbp, float* skT) {
  const bool vec = (reinterpret_cast<uintptr_t>(k16) & 15u) == 0;
  for (int b = threadIdx.x; b < NB; b += blockDim.x) {
    float kv[16];
    if (vec) {
      const uint4* src = reinterpret_cast<const uint4*>(k16 + (int64_t)b * 16);
      constexpr int kVec = 16 * (int)sizeof(T) / 16;
      uint4 u[kVec];
#pragma unroll
      for (int i = 0; i < kVec; ++i) u[i] = __ldg(src + i);
      const T* tv = reinterpret_cast<const T*>(u);
#pragma unroll
      for (int j = 0; j < 16; ++j) kv[j] = to_f32(tv[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) kv[j] = to_f32(k16[(int64_t)b * 16 + j]);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) skT[j * nbp + b] = kv[j];
  }
}

// Raw 16-D router projections x W_q^T of 16 tokens per CTA -> qraw [M, 16] (fp32).
// bf16 with D % 64 == 0: mma.sync over 64-element chunks of the hidden dimension, interleaved over the
// warps, partials summed in warp order.  Otherwise fp32 FFMA, two tokens per warp: lanes split the
// hidden dimension in 8-element vectors, then a butterfly sum.
// kW warps per CTA (mma form): 8, or 32 for batches of at most 64 tokens, whose projection is a chain of
// dependent loads per warp (D / 64 / kW chunks each) rather than a stream of x.
template <typename T, bool kMma, int kW = kRouteWarps>
__global__ void __launch_bounds__(kW * 32, kW == kRouteWarps ? 2 : 1)
route_proj_kernel(const T* __restrict__ x, const T* __restrict__ wq, int64_t M, int D, float* __restrict__ qraw) {
  constexpr int W = kMma ? kW : kRouteWarps, TPW = kProjTPW;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  griddep_launch_dependents();  // the routing kernel may launch; it waits for this grid before reading qraw
  const int64_t tok0 = (int64_t)blockIdx.x * kProjTokens;
  if constexpr (kMma) {
    __shared__ float part[W * 16 * 17];
    const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(x);
    const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(wq);
    const int g = lane >> 2, t = lane & 3;
    const int64_t ra = tok0 + g < M ? tok0 + g : M - 1;
    const int64_t rb = tok0 + g + 8 < M ? tok0 + g + 8 : M - 1;
    const __nv_bfloat16* pa = xb + ra * D + 16 * t;
    const __nv_bfloat16* pb = xb + rb * D + 16 * t;
    const __nv_bfloat16* qa = wb + (int64_t)g * D + 16 * t;
    const __nv_bfloat16* qb = wb + (int64_t)(8 + g) * D + 16 * t;
    float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
    const int nk = D / 64;
#pragma unroll 2
    for (int kc = warp; kc < nk; kc += W) {
      uint32_t A0[8], A1[8], B0[8], B1[8];
      const int k0 = kc * 64;
      ld32B(pa + k0, A0);
      ld32B(pb + k0, A1);
      ld32B(qa + k0, B0);
      ld32B(qb + k0, B1);
#pragma unroll
      for (int st = 0; st < 4; ++st) {
        mma_bf16_16816(c0, A0[2 * st], A1[2 * st], A0[2 * st + 1], A1[2 * st + 1], B0[2 * st], B0[2 * st + 1]);
        mma_bf16_16816(c1, A0[2 * st], A1[2 * st], A0[2 * st + 1], A1[2 * st + 1], B1[2 * st], B1[2 * st + 1]);
      }
    }
    // c0: projections 2t, 2t+1 of tokens g (c0[0..1]) and g+8 (c0[2..3]); c1: projections 8+2t, 9+2t
    float* q = part + warp * 16 * 17;
    q[g * 17 + 2 * t] = c0[0];
    q[g * 17 + 2 * t + 1] = c0[1];
    q[(g + 8) * 17 + 2 * t] = c0[2];
    q[(g + 8) * 17 + 2 * t + 1] = c0[3];
    q[g * 17 + 8 + 2 * t] = c1[0];
    q[g * 17 + 9 + 2 * t] = c1[1];
    q[(g + 8) * 17 + 8 + 2 * t] = c1[2];
    q[(g + 8) * 17 + 9 + 2 * t] = c1[3];
    __syncthreads();
    if (threadIdx.x < 256) {  // thread (r, j): projection j of token r, partials summed in warp order
      const int r = threadIdx.x >> 4, j = threadIdx.x & 15;
      float v = part[r * 17 + j];
#pragma unroll
      for (int w = 1; w < W; ++w) v += part[w * 16 * 17 + r * 17 + j];
      if (tok0 + r < M) qraw[(tok0 + r) * 16 + j] = v;
    }
  } else {
    float acc[TPW][16];
#pragma unroll
    for (int tt = 0; tt < TPW; ++tt)
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[tt][j] = 0.f;
    for (int c = lane * 8; c < D; c += 256) {
      float xv[TPW][8];
#pragma unroll
      for (int tt = 0; tt < TPW; ++tt) {
        const int64_t tk = tok0 + warp * TPW + tt;
        load8<T>(x + (tk < M ? tk : M - 1) * D + c, xv[tt]);
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float wv[8];
        load8<T>(wq + (int64_t)j * D + c, wv);
#pragma unroll
        for (int tt = 0; tt < TPW; ++tt)
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[tt][j] = fmaf(xv[tt][e], wv[e], acc[tt][j]);
      }
    }
#pragma unroll
    for (int tt = 0; tt < TPW; ++tt) {
      float mine = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float v = acc[tt][j];
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
        if (lane == j) mine = v;
      }
      const int64_t tk = tok0 + warp * TPW + tt;
      if (lane < 16 && tk < M) qraw[tk * 16 + lane] = mine;
    }
  }
}

// Persistent: each CTA stages the keys once, then routes groups of 16 tokens from their raw 16-D
// projections (route_proj_kernel).
template <typename T, int E>
__global__ void __launch_bounds__(kRouteWarps * 32, E <= 8 ? 3 : 1)
route_kernel(const RouteArgs a) {
  constexpr int TPW = kRouteTPW, N = 32 * E;
  griddep_launch_dependents();
  extern __shared__ float4 route_smem4[];
  char* smb = reinterpret_cast<char*>(route_smem4);
  const bool csr = a.key_cnt != nullptr;
  const RouteSmem L = route_smem(a.NB, a.nbl, E, a.hzero != nullptr, csr);
  const int nbp = (a.NB + 3) & ~3;
  float* skT = reinterpret_cast<float*>(smb + L.skT);       // [16][nbp] fp32 block keys, transposed
  int32_t* s_cnt = reinterpret_cast<int32_t*>(smb + L.cnt); // [nbl] group-local pairs per key
  int32_t* s_kb = reinterpret_cast<int32_t*>(smb + L.kbase);// [nbl] reserved start in the key bucket
  __shared__ float qsm[kRouteTokens][16];                   // raw 16-D projections of the group
  __shared__ int s_npair[kRouteTokens];
  __shared__ unsigned int s_ticket;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int NB = a.NB;
  const int64_t ngroups = (a.M + kRouteTokens - 1) / kRouteTokens;
  const uint64_t hrow = (uint64_t)a.hrow_vec * 16;

  const bool given = a.given_idx != nullptr;
  // ---- once per CTA: keys, the zero source of the H clears, the key counters
  if (!given) stage_keys<T>(static_cast<const T*>(a.k16), NB, nbp, skT);
  if (a.hzero) {
    uint4* z = reinterpret_cast<uint4*>(smb + L.zbuf);
    for (int i = threadIdx.x; i < (int)(kRouteZeroBytes / 16); i += blockDim.x) z[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  if (csr)
    for (int i = threadIdx.x; i < a.nbl; i += blockDim.x) s_cnt[i] = 0;
  // everything above reads only the block keys and this CTA's shared memory, so it overlaps the
  // projection kernel; the queries, the cleared counters and the previous call's readers of H are ordered
  // by this wait
  griddep_wait();  // the projection kernel's queries are complete and visible
  __syncthreads();

  for (int64_t grp = blockIdx.x; grp < ngroups; grp += gridDim.x) {
    const int64_t tok0 = grp * kRouteTokens;
    const int ntok = (int)((a.M - tok0) < kRouteTokens ? (a.M - tok0) : kRouteTokens);
    if (a.hzero && threadIdx.x == 0) {
      // the masked activations H must read zero for unselected (token, block) pairs: clear the group's
      // contiguous rows with bulk copies from the zero buffer while the warps route
      bulk_wait_read<2>();  // bound the clears in flight
      char* dst = reinterpret_cast<char*>(a.hzero) + (uint64_t)tok0 * hrow;
      const uint64_t total = (uint64_t)ntok * hrow;
      const uint32_t zs = smem_u32(smb + L.zbuf);
      for (uint64_t off = 0; off < total; off += kRouteZeroBytes) {
        const uint64_t rest = total - off;
        bulk_store(dst + off, zs, (uint32_t)(rest < kRouteZeroBytes ? rest : kRouteZeroBytes));
      }
      bulk_commit();
    }
    {  // this warp's tokens only (other warps may already be working on theirs): lane (tt, j)
      const int r = warp * TPW + (lane >> 4);
      if (!given && lane < 16 * TPW && tok0 + r < a.M) qsm[r][lane & 15] = __ldcg(&a.qraw[(tok0 + r) * 16 + (lane & 15)]);
      if (lane < TPW) s_npair[warp * TPW + lane] = 0;
    }
    __syncwarp();

    // ---- per token: RMSNorm, scores, selection, group-local CSR entries
    float* pbuf = reinterpret_cast<float*>(smb + L.pbuf) + warp * N;
    int32_t* sbuf = reinterpret_cast<int32_t*>(smb + L.sbuf) + warp * N;
    const float eps = 1.1920928955078125e-07f;  // torch.finfo(float32).eps: F.rms_norm's default
#pragma unroll 1
    for (int tt = 0; tt < TPW; ++tt) {
      const int r = warp * TPW + tt;
      const int64_t tok = tok0 + r;
      if (tok >= a.M) break;
      if (given) {
        // the token's route, computed by another rank: its remote ids into sbuf
        const int cmax = a.given_cap < NB - a.sel.base ? a.given_cap : NB - a.sel.base;  // fits sbuf / plist
        int c = __ldg(&a.given_cnt[tok]);
        c = c < 0 ? 0 : (c > cmax ? cmax : c);
        if (csr) {
          for (int i = lane; i < c; i += 32) sbuf[i] = __ldg(&a.given_idx[tok * a.given_cap + i]);
          __syncwarp();
          int32_t* pl = reinterpret_cast<int32_t*>(smb + L.plist) + r * N;
          const int npair = a.sel.base + c;
          for (int sl = lane; sl < npair; sl += 32) {
            const int b = sl < a.sel.base ? sl : sbuf[sl - a.sel.base];
            int e = -1;
            if (b < 0 || b >= NB) {
              record_error(a.err, kErrBadTile);  // a given id outside the blocks: reported, skipped
            } else if (b % a.stride == a.offset) {
              const int kl = b / a.stride;
              const int pos = atomicAdd(&s_cnt[kl], 1);
              if (pos < 16) e = (kl << 4) | pos;  // a block listed twice by the group's tokens could exceed
              else record_error(a.err, kErrBadTile);  // the 16 positions of an entry: reported, skipped
            }
            pl[sl] = e;
          }
          if (lane == 0) s_npair[r] = npair;
        }
        __syncwarp();  // sbuf is rewritten by the next token of this warp
        continue;
      }
      float qn[16];
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        qn[j] = qsm[r][j];
        ss = fmaf(qn[j], qn[j], ss);
      }
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(ss * (1.0f / 16.0f) + eps));
      float qown = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (lane == j) qown = qn[j];
        qn[j] *= inv;
      }
      if (a.q16 && lane < 16) a.q16[tok * 16 + lane] = qown * inv;
      float s[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int b = e * 32 + lane;
        float sc = -INFINITY;
        if (b < NB) {
          float acc = 0.f;
#pragma unroll
          for (int j = 0; j < 16; ++j) acc = fmaf(qn[j], skT[j * nbp + b], acc);
          acc *= 0.25f;  // / sqrt(16): exact power-of-two scaling
          if (a.scores) a.scores[tok * NB + b] = acc;
          sc = a.temperature != 1.0f ? __fdiv_rn(acc, a.temperature) : acc;
        }
        s[e] = sc;
      }
      const int counts = select_token<E>(s, tok, a.sel, pbuf, csr ? sbuf : nullptr, skT, nbp, lane);
      if (csr) {
        __syncwarp();
        // pair list entry: (local key << 4) | position among this group's tokens of that key, or -1
        int32_t* pl = reinterpret_cast<int32_t*>(smb + L.plist) + r * N;
        const int npair = a.sel.base + counts;
        for (int sl = lane; sl < npair; sl += 32) {
          const int b = sl < a.sel.base ? sl : sbuf[sl - a.sel.base];
          int e = -1;
          if (b % a.stride == a.offset) {
            const int kl = b / a.stride;
            e = (kl << 4) | atomicAdd(&s_cnt[kl], 1);
          }
          pl[sl] = e;
        }
        if (lane == 0) s_npair[r] = npair;
      }
      __syncwarp();  // pbuf / sbuf are rewritten by the next token of this warp
    }

    __syncthreads();  // qsm, part, the pair lists and the key counters of the group are complete
    if (csr) {
      // one global reservation per key for the group's tokens (all in one token chunk), then the scatter
      const int64_t kb = (tok0 / a.chunk) * a.nbl;
      for (int k = threadIdx.x; k < a.nbl; k += blockDim.x) {
        const int c = s_cnt[k];
        s_kb[k] = c ? atomicAdd(&a.key_cnt[kb + k], c) : 0;
        s_cnt[k] = 0;  // ready for the next group
      }
      __syncthreads();
#pragma unroll 1
      for (int tt = 0; tt < TPW; ++tt) {
        const int r = warp * TPW + tt;
        const int32_t* pl = reinterpret_cast<const int32_t*>(smb + L.plist) + r * N;
        const int npair = s_npair[r];
        for (int sl = lane; sl < npair; sl += 32) {
          const int e = pl[sl];
          if (e >= 0) {
            const int kl = e >> 4;
            const int64_t pos = (int64_t)s_kb[kl] + (e & 15);
            if (pos < a.key_cap) a.pair_tok[(kb + kl) * a.key_cap + pos] = (int32_t)(tok0 + r);
            else record_error(a.err, kErrBadTile);
          }
        }
      }
      __syncthreads();  // s_kb and the pair lists are reused by the next group
    }
  }

  if (csr) {
    // the last CTA to finish turns the key counts into the gate/up tile list
    if (threadIdx.x == 0) {
      __threadfence();
      s_ticket = atomicAdd(a.ticket, 1u);
    }
    __syncthreads();
    if (s_ticket == gridDim.x - 1) {
      __threadfence();
      build_tile_list(a);
    }
  }
  if (a.hzero && threadIdx.x == 0) bulk_wait_all();  // the H clears complete before the CTA retires
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
                         int NB, float temperature, float* scores, float* q16, cudaStream_t st,
                         const float* kcos) {
  if (M <= 0) return FP_OK;
  if (dtype == FP_DTYPE_BF16 && D % (64 * kMmaWarps) == 0 && temperature == 1.0f) {
    const size_t smem = (size_t)NB * 16 * sizeof(float) + kMmaWarps * 16 * 17 * sizeof(float);
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(router_scores_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
      return FP_ERR_CUDA;
    const int blocks = (int)((M + 15) / 16);
    router_scores_mma_kernel<<<blocks, kMmaWarps * 32, smem, st>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)wq, (const __nv_bfloat16*)k16, M, D, NB, scores, q16, kcos);
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
        temperature, scores, q16, kcos);
  else
    router_scores_kernel<float><<<blocks, kScoreWarps * 32, smem, st>>>(
        (const float*)x, (const float*)wq, (const float*)k16, M, D, NB, 0.25f, temperature, scores, q16, kcos);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

template <int E>
int select_go(const float* scores, int64_t M, float temperature, const SelectOut& o, const float* k16f,
              cudaStream_t st) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t need = (M + kSelWarps - 1) / kSelWarps;
  const int blocks = (int)std::min<int64_t>(need, (int64_t)sms * 8);
  const size_t smem = (size_t)kSelWarps * 32 * E * sizeof(float) + (o.ctx16 ? (size_t)o.NB * 16 * sizeof(float) : 0);
  if (ensure_smem<select_blocks_kernel<E>>(smem) != FP_OK) return FP_ERR_CUDA;
  select_blocks_kernel<E><<<blocks, kSelWarps * 32, smem, st>>>(scores, M, temperature, o, k16f);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

int launch_select(const float* scores, int64_t M, int NB, int base, float top_p, int k_min, int k_max,
                  int capacity, float temperature, int32_t* idx, int32_t* cnt, const float* k16f,
                  float* ctx16, float* stats, cudaStream_t st) {
  const SelectOut o{NB, base, top_p, k_min, k_max, capacity, idx, cnt, ctx16, stats};
  return launch_select_out(scores, M, temperature, o, k16f, st);
}

int launch_select_out(const float* scores, int64_t M, float temperature, const SelectOut& o, const float* k16f,
                      cudaStream_t st) {
  if (M <= 0) return FP_OK;
  const int NB = o.NB;
  if (NB <= 32) return select_go<1>(scores, M, temperature, o, k16f, st);
  if (NB <= 64) return select_go<2>(scores, M, temperature, o, k16f, st);
  if (NB <= 128) return select_go<4>(scores, M, temperature, o, k16f, st);
  if (NB <= 256) return select_go<8>(scores, M, temperature, o, k16f, st);
  if (NB <= 512) return select_go<16>(scores, M, temperature, o, k16f, st);
  if (NB <= 1024) return select_go<32>(scores, M, temperature, o, k16f, st);
  return FP_ERR_UNSUPPORTED;
}

template <typename T, int E>
int route_go(const RouteArgs& a, bool mma, cudaStream_t st) {
  const int64_t pblocks = (a.M + kProjTokens - 1) / kProjTokens;
  const int64_t groups = (a.M + kRouteTokens - 1) / kRouteTokens;
  if (a.given_idx) {
    // routes given: no projection; the routing kernel builds the block lists only
  } else if (mma) {
    if (a.M <= 64)
      route_proj_kernel<__nv_bfloat16, true, 32><<<(unsigned)pblocks, 32 * 32, 0, st>>>(
          static_cast<const __nv_bfloat16*>(a.x), static_cast<const __nv_bfloat16*>(a.wq), a.M, a.D, a.qraw);
    else
      route_proj_kernel<__nv_bfloat16, true><<<(unsigned)pblocks, kRouteWarps * 32, 0, st>>>(
          static_cast<const __nv_bfloat16*>(a.x), static_cast<const __nv_bfloat16*>(a.wq), a.M, a.D, a.qraw);
  }
  else
    route_proj_kernel<T, false><<<(unsigned)pblocks, kRouteWarps * 32, 0, st>>>(
        static_cast<const T*>(a.x), static_cast<const T*>(a.wq), a.M, a.D, a.qraw);
  if (cudaGetLastError() != cudaSuccess) return FP_ERR_CUDA;
  const size_t smem = (size_t)route_smem(a.NB, a.nbl, E, a.hzero != nullptr, a.key_cnt != nullptr).total;
  if (ensure_smem<route_kernel<T, E>>(smem) != FP_OK) return FP_ERR_CUDA;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, route_kernel<T, E>, kRouteWarps * 32, smem) !=
      cudaSuccess)
    return FP_ERR_CUDA;
  const int64_t blocks = std::min<int64_t>(groups, (int64_t)std::max(per_sm, 1) * std::max(a.num_sms, 1));
  return launch_pdl(route_kernel<T, E>, dim3((unsigned)blocks), dim3(kRouteWarps * 32), smem, st, a) == cudaSuccess
             ? FP_OK : FP_ERR_CUDA;
}

template <int E>
int route_dtype(const RouteArgs& a, int dtype, cudaStream_t st) {
  if (dtype == FP_DTYPE_F32) return route_go<float, E>(a, false, st);
  return route_go<__nv_bfloat16, E>(a, a.D % 64 == 0, st);
}

int launch_route(const RouteArgs& a, int dtype, cudaStream_t st) {
  if (a.M <= 0) return FP_OK;
  if (dtype != FP_DTYPE_F32 && dtype != FP_DTYPE_BF16) return FP_ERR_UNSUPPORTED;
  if (a.NB <= 32) return route_dtype<1>(a, dtype, st);
  if (a.NB <= 64) return route_dtype<2>(a, dtype, st);
  if (a.NB <= 128) return route_dtype<4>(a, dtype, st);
  if (a.NB <= 256) return route_dtype<8>(a, dtype, st);
  if (a.NB <= 512) return route_dtype<16>(a, dtype, st);
  if (a.NB <= 1024) return route_dtype<32>(a, dtype, st);
  return FP_ERR_UNSUPPORTED;
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

static int pow2_at_least(int n) {
  int p = 32;
  while (p < n) p <<= 1;
  return p;
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
