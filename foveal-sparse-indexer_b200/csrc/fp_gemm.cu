// Tensor-core (tcgen05 / TMEM / TMA) kernels of the gated Pattention contraction, bf16 in, fp32 accumulate.
//
//   gate/up:  for each work tile (parameter block b, up to 256 tokens that selected b):
//             D[128 x n] = [K_gate,b ; K_up,b] (128 x D) . X[tokens]^T (D x n)   (A = weights, B = tokens)
//             h[t, c] = silu(D[gate c, t]) * D[up c, t]  ->  H[t, slot(b)*64 + c]  (bf16)
//   down:     Y[tokens x 256 cols] = sum over k-blocks j of H[:, j*64:+64] . V_b(j)^T ; + ctx16 . W_out^T
//             on CTA pairs (cta_group::2, 256-token tiles) from 256 tokens up, on one SM below
//   energy:   the gate/up kernel with an fp32 |h| reduction per (token, block) instead of writing H
//             (teacher block energies of the offline calibration)
//   mapped:   the down kernels in a block-mapped form for the union contractions of BlockSparseLinear and
//             the Tokenformer layers: B rows and Y columns through per-64-column block maps, tile and
//             k-loop bounds from device counts, bias in the epilogue (DownArgs.nmap / omap / ncnt / kcnt)
//
// Reference semantics: foveal_indexer/foveal_pattention.py:329-335 (two projections, SwiGLU, V
// projection over the active blocks), per-token form foveal_indexer/pattention_triton.py:280-311,
// additive stream foveal_pattention.py:338-342.
//
// All kernels are persistent (one CTA per SM) and warp-specialised: warp 0 issues TMA loads into a
// shared-memory ring (gate/up: plus 16 cp.async warps gathering token rows), warp 1 (one thread)
// issues tcgen05.mma into one of two TMEM accumulators (2 x 256 fp32 columns), warps 2-5 drain the
// other accumulator (the epilogue overlaps the next tile's MMAs).  Operand tiles are K-major with the
// 128-byte swizzle: one 64-element k-block is exactly one parameter block's worth of the contraction
// dimension of the down projection.
#include "fp_internal.cuh"

#include <cudaTypedefs.h>
#include <cstring>
#include <mutex>

namespace fp {

constexpr uint32_t kABytes = kTileM * kTileK * 2;  // 16 KB
constexpr uint32_t kBBytes = kTileN * kTileK * 2;  // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kTmemCols = 512;

template <int S>
struct __align__(8) PipeBarsT {
  static constexpr int kStagesN = S;
  uint64_t full[S];
  uint64_t empty[S];
  uint64_t accf[2];
  uint64_t acce[2];
  uint64_t done;
  uint32_t tmem;
  int32_t consumed;
};
using PipeBars = PipeBarsT<kStages>;     // down kernel
constexpr size_t kGemmSmem = 1024 + kStages * kStageBytes + sizeof(PipeBars) + 64;

// Gate/up kernel configurations: at most NMAX tokens per tile and STAGES shared-memory stages of
// 16 KB (weights) + NMAX x 128 B (token rows).  <256, 4> in general; <64, 8> for batches of at most 64
// tokens (decode), whose tiles are small and whose time is the streaming of the blocks' weights: twice
// the stages keep twice the bytes in flight per SM.
template <int NMAX, int STAGES, int GATHER_WARPS>
struct GuCfg {
  static constexpr int kN = NMAX;
  static constexpr int kS = STAGES;
  // token-row gather warps (cp.async), warps 6..; fewer for small tiles leaves each thread more registers
  static constexpr int kGatherThreads = 32 * GATHER_WARPS;
  static constexpr int kThreads = 192 + kGatherThreads;
  using Bars = PipeBarsT<STAGES>;
  static constexpr uint32_t kBBytes = NMAX * kTileK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr size_t kSmem = 1024 + STAGES * kStageBytes + sizeof(Bars) + 64;
  static_assert(kSmem <= 227 * 1024, "gate/up shared memory");
};
using GuBig = GuCfg<kGuN, kGuStages, 16>;
using GuSmall = GuCfg<64, 8, 8>;

__device__ __forceinline__ uint8_t* aligned_smem(uint8_t* raw) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
}

// Sum over splits of 4 consecutive fp32 partials at element offset `off` (stride `n` between splits), in
// split order; the loads of up to 8 splits are issued before the first add (decode-size reductions are
// bound by load latency, not bandwidth).
__device__ __forceinline__ float4 splitk_sum4(const float* __restrict__ part, int ks, int64_t n, int64_t off) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k0 = 0; k0 < ks; k0 += 8) {
    float4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (k0 + j < ks) v[j] = __ldcg(reinterpret_cast<const float4*>(part + (int64_t)(k0 + j) * n + off));
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (k0 + j < ks) {
        if (k0 + j == 0) {
          acc = v[j];
        } else {
          acc.x += v[j].x; acc.y += v[j].y; acc.z += v[j].z; acc.w += v[j].w;
        }
      }
  }
  return acc;
}

__device__ __forceinline__ void store4(void* out, int64_t idx, float4 s, int out_f32) {
  if (out_f32) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + idx) = s;
  } else {
    const __nv_bfloat162 a = __floats2bfloat162_rn(s.x, s.y), b = __floats2bfloat162_rn(s.z, s.w);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(out) + idx) = u;
  }
}

// Lane 0 waits, the warp follows its verdict (keeps warp-collective instructions uniform).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, err, code);
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  __syncwarp();
  return ok;
}

template <class Bars>
__device__ __forceinline__ void pipe_init(Bars* bars, int epi_warps, int full_count = 1) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < Bars::kStagesN; ++s) {
      mbar_init(&bars->full[s], full_count);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->accf[a], 1);
      mbar_init(&bars->acce[a], epi_warps);
    }
    mbar_init(&bars->done, 1);
    bars->consumed = 0;
    fence_mbar_init();
  }
  if ((threadIdx.x >> 5) == 0) {
    tmem_alloc(&bars->tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

// After every role has left its loop: make sure no TMA copy or MMA is still in flight, then free TMEM.
template <class Bars>
__device__ __forceinline__ void pipe_teardown(Bars* bars, uint32_t issued, int* err) {
  constexpr int S = Bars::kStagesN;
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && aborted(err)) {
    for (uint32_t i = (uint32_t)bars->consumed; i < issued; ++i)
      if (!mbar_wait(&bars->full[i % S], (i / S) & 1u, nullptr, 0)) {
        record_error(err, kErrDrain);
        break;
      }
  }
  __syncthreads();
  if ((threadIdx.x >> 5) == 0) {
    tc_fence_after();
    tmem_dealloc(bars->tmem, kTmemCols);
  }
}

// MMA issuer tail: wait until every tcgen05.mma issued by this thread has completed.
template <class Bars>
__device__ __forceinline__ void mma_quiesce(Bars* bars, uint32_t consumed, int* err) {
  bars->consumed = (int32_t)consumed;
  umma_commit(&bars->done);
  if (!mbar_wait(&bars->done, 0, nullptr, 0)) record_error(err, kErrDrain);
}

// ============================================================================================
// Gate/up grouped GEMM with SwiGLU epilogue
// ============================================================================================
struct GuTile {
  int b;               // global parameter block
  int slot;            // column slot in H (x64)
  const int32_t* list; // token ids (nullptr: identity r0 + i)
  int64_t r0;
  int n;               // valid tokens in this tile (0: skip)
};

template <int NMAX>
__device__ __forceinline__ GuTile gu_decode(const GateUpArgs& a, int tile) {
  GuTile t;
  if (a.tiles) {
    const int2 d = a.tiles[tile];
    const int key = d.x;
    t.slot = key % a.nbl;
    t.b = t.slot * a.stride + a.offset;
    const int cnt = a.key_cnt[key];
    t.list = a.pair_tok + (int64_t)key * a.key_cap + d.y;
    t.r0 = d.y;
    t.n = min(balanced_rows(cnt), cnt - d.y);
  } else {
    const int key = tile % a.n_keys;  // token-tile-major order: concurrent tiles share rows of x
    const int64_t rt = tile / a.n_keys;
    t.slot = key;
    t.b = a.active[key];
    t.list = nullptr;
    t.r0 = rt * NMAX;
    t.n = (int)((a.M - t.r0) < (int64_t)NMAX ? (a.M - t.r0) : (int64_t)NMAX);
  }
  if (t.b < 0 || (int64_t)(t.b + 1) * kBlock > a.Np) {
    record_error(a.err, kErrBadTile);
    t.n = 0;
  }
  return t;
}

// Token of row i of a tile.  Listed ids outside [0, M) (a corrupt work list) are reported and returned as
// -1: the gathers then read token 0's row and the epilogue skips the store, so no access leaves x or H.
__device__ __forceinline__ int gu_token(const GuTile& t, int i, const GateUpArgs& a) {
  if (!t.list) return (int)(t.r0 + i);
  const int tok = t.list[i];
  if ((unsigned)tok >= (unsigned long long)a.M) {
    record_error(a.err, kErrBadTile);
    return -1;
  }
  return tok;
}

// Activation of one 32-column chunk of a gate/up accumulator read from TMEM and its store into H (or the
// energy partials).  Warp quarter q, lane L: v = TMEM lane 32q + L (packed row: gate channel 16q + L for
// L < 16, up channel 16q + L - 16 otherwise) over 32 token columns; tok_l = token of column L of the chunk
// (-1: none).  Lanes L and L + 16 exchange halves so that each computes h for 16 of the 32 tokens.
__device__ __forceinline__ void gu_store_chunk(const GateUpArgs& a, const uint32_t (&v)[32], int tok_l, int slot,
                                               int q, int lane) {
  __nv_bfloat16* hbase = reinterpret_cast<__nv_bfloat16*>(a.h) + (int64_t)slot * kBlock + 16 * q + (lane & 15);
  const bool swiglu = a.act == FP_ACT_SWIGLU;  // uniform: the SwiGLU loop carries no activation switch
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint32_t send = lane < 16 ? v[16 + j] : v[j];
    const float recv = __uint_as_float(__shfl_xor_sync(0xffffffffu, send, 16));
    const float gv = lane < 16 ? __uint_as_float(v[j]) : recv;
    const float u = lane < 16 ? recv : __uint_as_float(v[16 + j]);
    const float h = swiglu ? __fdividef(gv, 1.0f + __expf(-gv)) * u : pattention_act<false>(a.act, gv, u);
    const int tok = __shfl_sync(0xffffffffu, tok_l, lane < 16 ? j : 16 + j);
    if (a.energy) {
      // |h| summed over this half-warp's 16 channels (fixed order), one partial per TMEM quarter
      float e = fabsf(h);
      e += __shfl_xor_sync(0xffffffffu, e, 8);
      e += __shfl_xor_sync(0xffffffffu, e, 4);
      e += __shfl_xor_sync(0xffffffffu, e, 2);
      e += __shfl_xor_sync(0xffffffffu, e, 1);
      if ((lane & 15) == 0 && tok >= 0) a.energy[((int64_t)q * a.M + tok) * a.nbl + slot] = e;
    } else if (tok >= 0) {
      hbase[(int64_t)tok * a.ldh] = __float2bfloat16_rn(h);
    }
  }
}


template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads, 1)
gateup_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
              const GateUpArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = aligned_smem(smem_raw);
  constexpr int kN = Cfg::kN, kS = Cfg::kS;
  constexpr uint32_t kStage = Cfg::kStageBytes;
  constexpr int kGatherThreads = Cfg::kGatherThreads;
  constexpr int kRowsPerGatherThread = kN * 8 / kGatherThreads;  // 16-byte chunks per thread per stage
  static_assert(kRowsPerGatherThread * kGatherThreads == kN * 8, "gather split");
  using Bars = typename Cfg::Bars;
  Bars* bars = reinterpret_cast<Bars*>(smem + kS * kStage);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool gathered = a.tiles != nullptr;  // token lists (cp.async gathers) or identity rows (TMA box)

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
  }
  // full barrier: one expect_tx arrival (TMA) + one arrival per gather thread
  pipe_init(bars, 4, 1 + kGatherThreads);
  if (kN == 64 && a.pf.n > 0) {
    // while the routing kernel runs: this CTA's share of the L2 prefetch, 64 KB pieces dealt round-robin
    // over the CTAs (each SM's copy engine generates only its share of the requests)
    constexpr int64_t kPiece = 64 * 1024;
    const int64_t per_run = (a.pf.bytes + kPiece - 1) / kPiece;
    const int64_t total = per_run * a.pf.n;
    for (int64_t i = blockIdx.x + (int64_t)threadIdx.x * gridDim.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t run = i / per_run, off = (i - run * per_run) * kPiece;
      const int64_t len = a.pf.bytes - off < kPiece ? a.pf.bytes - off : kPiece;
      bulk_prefetch_l2(a.pf.base + run * a.pf.stride + off, (uint32_t)len);
    }
  }
  griddep_wait();  // the routing kernel's work list, token lists and cleared H are complete
  griddep_launch_dependents();
  const uint32_t tmem_base = bars->tmem;
  const int ntiles = gathered ? a.meta[0] : a.n_keys * (int)((a.M + kN - 1) / kN);
  const int nkb = a.D / kTileK;
  const int nbt = a.Np / kBlock;  // blocks of the packed weight (tile kb * nbt + b)
  // work units: tile u / ks over k-blocks [kr0(u), kr1(u)) (ks = 1: whole tiles; the split exists only
  // in the configuration for batches of at most 64 tokens)
  const int ks = (kN == 64 && a.gu_ks > 1) ? a.gu_ks : 1;
  const int nunits = ntiles * ks;
  auto kr0 = [&](int u) { return (u % ks) * nkb / ks; };
  auto kr1 = [&](int u) { return (u % ks + 1) * nkb / ks; };
  uint32_t issued = 0;

  if (warp == 0) {
    // ---------------- TMA producer: packed gate/up weight tile (one 128-row box per stage) and, for
    // identity token ranges, the x tile (one 256-row box)
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      // batches of at most 64 tokens read every weight tile once: keep it from evicting the partials,
      // H and x from L2
      const uint64_t pol = l2_policy_evict_first();
      for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
        const GuTile t = gu_decode<kN>(a, u / ks);
        if (t.n <= 0) continue;
        for (int kb = kr0(u); kb < kr1(u); ++kb, ++it) {
          const int s = it % kS;
          const uint32_t ph = (it / kS) & 1u;
          if (!mbar_wait(&bars->empty[s], ph ^ 1u, a.err, kErrWaitEmpty)) { ok = false; break; }
          uint8_t* As = smem + s * kStage;
          mbar_arrive_expect_tx(&bars->full[s], kABytes + (gathered ? 0u : Cfg::kBBytes));
          if (kN == 64)
            tma_load_2d_hint(As, &tm_w, &bars->full[s], 0, (kb * nbt + t.b) * kTileM, pol);
          else
            tma_load_2d(As, &tm_w, &bars->full[s], 0, (kb * nbt + t.b) * kTileM);
          if (!gathered) tma_load_2d(As + kABytes, &tm_x, &bars->full[s], kb * kTileK, (int)t.r0);
        }
      }
      issued = it;
    }
    __syncwarp();
  } else if (warp >= 6) {
    // ---------------- token-row gathers: thread g copies 16-byte chunk (g % 8) of rows g/8 + kRowStep*j,
    // written in the 128-byte swizzle pattern TMA would use (chunk c of row r at c ^ (r % 8))
    constexpr int kRowStep = kGatherThreads / 8;  // rows covered by one pass of the gather threads
    const int g = threadIdx.x - 192;
    const int chunk = g & 7, row0 = g >> 3;
    const uint32_t swz = (uint32_t)((chunk ^ (row0 & 7)) << 4);  // kRowStep is a multiple of 8
    const char* xbytes = reinterpret_cast<const char*>(a.x);
    uint32_t it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
      const GuTile t = gu_decode<kN>(a, u / ks);
      if (t.n <= 0) continue;
      const int npad = (t.n + 15) & ~15;
      int64_t src[kRowsPerGatherThread];
#pragma unroll
      for (int j = 0; j < kRowsPerGatherThread; ++j) {
        const int r = row0 + kRowStep * j;
        const int tl = (gathered && r < npad) ? gu_token(t, r < t.n ? r : t.n - 1, a) : 0;
        const int tok = tl < 0 ? 0 : tl;
        src[j] = (int64_t)tok * a.D * 2 + chunk * 16;
      }
      for (int kb = kr0(u); kb < kr1(u); ++kb, ++it) {
        const int s = it % kS;
        const uint32_t ph = (it / kS) & 1u;
        if (!warp_wait(&bars->empty[s], ph ^ 1u, a.err, kErrWaitEmpty)) { ok = false; break; }
        if (gathered) {
          const uint32_t bs = smem_u32(smem + s * kStage + kABytes) + swz;
          const int64_t koff = (int64_t)kb * kTileK * 2;
#pragma unroll
          for (int j = 0; j < kRowsPerGatherThread; ++j) {
            const int r = row0 + kRowStep * j;
            if (r < npad) cp_async_16(bs + r * 128, xbytes + src[j] + koff);
          }
        }
        cp_async_arrive_noinc(&bars->full[s]);
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // no copy of this thread outlives the CTA
  } else if (warp == 1) {
    // ---------------- MMA issuer (one thread)
    if (lane == 0) {
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
        const GuTile t = gu_decode<kN>(a, u / ks);
        if (t.n <= 0) continue;
        const int npad = (t.n + 15) & ~15;
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(&bars->acce[acc], aph ^ 1u, a.err, kErrWaitAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kTileN;
        const uint32_t idesc = umma_idesc_bf16(kTileM, npad);
        const int k0 = kr0(u);
        for (int kb = k0; kb < kr1(u); ++kb) {
          const int s = it % kS;
          const uint32_t ph = (it / kS) & 1u;
          if (!mbar_wait(&bars->full[s], ph, a.err, kErrWaitFull)) { ok = false; break; }
          fence_proxy_async_smem();
          tc_fence_after();
          const uint64_t ad = umma_desc_sw128(smem_u32(smem + s * kStage));
          const uint64_t bd = umma_desc_sw128(smem_u32(smem + s * kStage + kABytes));
#pragma unroll
          for (int k = 0; k < kTileK / 16; ++k)
            umma_bf16(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb != k0) || k != 0);
          umma_commit(&bars->empty[s]);
          ++it;
        }
        if (!ok) break;
        umma_commit(&bars->accf[acc]);
        ++local;
      }
      mma_quiesce(bars, it, a.err);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: warps 2..5; warp w reads TMEM lanes [32*(w%4), +32)
    const int q = warp & 3;
    int local = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
      const int tile = u / ks;
      const GuTile t = gu_decode<kN>(a, tile);
      if (t.n <= 0) continue;
      const int npad = (t.n + 15) & ~15;
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!warp_wait(&bars->accf[acc], aph, a.err, kErrWaitAccFull)) break;
      tc_fence_after();
      if (kN != 64 || ks == 1) {
        for (int c = 0; c * 32 < npad; ++c) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld32(tmem_base + acc * kTileN + c * 32 + ((uint32_t)(32 * q) << 16), v);
          tmem_ld_wait();
          const int ni = c * 32 + lane;
          gu_store_chunk(a, v, ni < t.n ? gu_token(t, ni, a) : -1, t.slot, q, lane);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->acce[acc]);
      } else {
        // split unit: this quarter's fp32 rows (row 32q + lane, npad token columns) to the unit's slot;
        // gateup_split_combine_kernel sums a tile's slots and runs the activation
        const int64_t row = 32 * q + lane;
        float* mine = a.gu_part + (((int64_t)tile * ks + u % ks) * kTileM + row) * kN;
        for (int c = 0; c * 32 < npad; ++c) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld32(tmem_base + acc * kTileN + c * 32 + ((uint32_t)(32 * q) << 16), v);
          tmem_ld_wait();
          float4* dst = reinterpret_cast<float4*>(mine + c * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            dst[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                 __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->acce[acc]);
      }
      ++local;
    }
  }
  pipe_teardown(bars, issued, a.err);
}

// Second half of the split gate/up (batches of at most 64 tokens): per tile, the fp32 partials of its
// gu_ks work units are summed in split order into shared memory (coalesced loads, all splits in flight),
// then each thread computes h for one (token, channel) and the CTA stores whole 128-byte rows of H.
// Packed row of gate channel c: 32 (c / 16) + c % 16; of up channel c: that + 16.
constexpr int kGuCombineThreads = 1024;  // a base block's tile (64 tokens) is 2048 float4 of partials per split
__global__ void __launch_bounds__(kGuCombineThreads) gateup_split_combine_kernel(const GateUpArgs a) {
  constexpr int kN = 64;
  __shared__ float s_acc[kTileM][kN + 1];
  __shared__ int s_tok[kN];
  // The work list and token lists were written by the routing kernel, which completed before the gate/up
  // kernel passed its own wait, i.e. before this grid was launched: they are read before the wait for the
  // gate/up partials, off the critical path.  (A CTA with a second tile reads it after the wait.)
  const int ks = a.gu_ks;
  const int ntiles = a.meta[0];
  const bool swiglu = a.act == FP_ACT_SWIGLU;
  GuTile t0{};
  int tok0 = -1;
  if (blockIdx.x < ntiles) {
    t0 = gu_decode<kN>(a, blockIdx.x);
    if (threadIdx.x < t0.n) tok0 = gu_token(t0, threadIdx.x, a);
  }
  griddep_wait();  // every unit's partial is stored
  griddep_launch_dependents();
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const bool first = tile == (int)blockIdx.x;
    const GuTile t = first ? t0 : gu_decode<kN>(a, tile);
    if (t.n <= 0) continue;  // uniform over the CTA
    const int npad = (t.n + 15) & ~15;
    const int nq = npad / 4;  // float4 per row
    if (threadIdx.x < t.n) s_tok[threadIdx.x] = first ? tok0 : gu_token(t, threadIdx.x, a);
    const float4* part = reinterpret_cast<const float4*>(a.gu_part + (int64_t)tile * ks * kTileM * kN);
    for (int i = threadIdx.x; i < kTileM * nq; i += kGuCombineThreads) {
      const int row = i / nq, c4 = i - row * nq;
      const int64_t off = (int64_t)row * (kN / 4) + c4;
      const float4 v = splitk_sum4(reinterpret_cast<const float*>(part), ks, (int64_t)kTileM * kN, 4 * off);
      s_acc[row][4 * c4] = v.x; s_acc[row][4 * c4 + 1] = v.y;
      s_acc[row][4 * c4 + 2] = v.z; s_acc[row][4 * c4 + 3] = v.w;
    }
    __syncthreads();
    __nv_bfloat16* hbase = reinterpret_cast<__nv_bfloat16*>(a.h) + (int64_t)t.slot * kBlock;
    for (int i = threadIdx.x; i < t.n * kBlock; i += kGuCombineThreads) {
      const int tc = i / kBlock, ch = i - tc * kBlock;
      const int grow = 32 * (ch >> 4) + (ch & 15);
      const float gv = s_acc[grow][tc], u = s_acc[grow + 16][tc];
      const float h = swiglu ? __fdividef(gv, 1.0f + __expf(-gv)) * u : pattention_act<false>(a.act, gv, u);
      const int tok = s_tok[tc];
      if (tok >= 0) hbase[(int64_t)tok * a.ldh + ch] = __float2bfloat16_rn(h);
    }
    __syncthreads();  // s_acc and s_tok are rewritten by the CTA's next tile
  }
}

// Packed gate/up layout of one parameter block b (128 rows): rows 32q .. 32q+15 are gate channels
// 16q .. 16q+15 and rows 32q+16 .. 32q+31 the up channels 16q .. 16q+15 (q = 0..3), so that after the
// MMA (A = these rows) each 32-lane TMEM quarter holds the gate and up values of the same 16 channels.
// Tile-contiguous: the 128 rows x 64 columns [kb*64, +64) of block b that one pipeline stage loads are
// one contiguous 16 KB tile, so every TMA box streams whole DRAM pages instead of 128 bytes from each of
// 128 rows D * 2 bytes apart.  Tiles are k-block-major (tile index kb * NB + b): the 64 tiles of one block
// lie NB tiles apart, spread over the whole packed region, so that a CTA streaming one block (decode
// tiles) reads from all of the memory evenly.
__global__ void pack_gate_up_kernel(const uint4* __restrict__ kg, const uint4* __restrict__ ku, int64_t rows,
                                    int vec_per_row, uint4* __restrict__ wgu) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // over 2*rows*vec_per_row 16-byte words
  if (i >= 2 * rows * vec_per_row) return;
  const int64_t NB = rows / 64;
  const int c = (int)(i & 7);            // 8 words = one 64-element row of a tile
  const int r = (int)((i >> 3) & 127);   // packed row inside the block
  const int64_t t = i >> 10;             // tile = kb * NB + b
  const int kb = (int)(t / NB);
  const int64_t b = t - (int64_t)kb * NB;
  const int q = r >> 5, w = r & 31;
  const int64_t src_row = b * 64 + 16 * q + (w & 15);
  wgu[i] = (w < 16 ? kg : ku)[src_row * vec_per_row + kb * 8 + c];
}

// V^T in tile-contiguous form for the down projection: the 256 output columns [n*256, +256) x 64
// parameter tokens of block gb that one stage loads are one contiguous 32 KB tile (rows = output columns,
// 64 elements each), tile index n * NB + gb; columns past D are zero.  One CTA transposes one tile
// through shared memory (v rows of 512 contiguous bytes in, 128-byte tile rows out).
__global__ void __launch_bounds__(256) pack_vt_kernel(const __nv_bfloat16* __restrict__ v, int D, int NB,
                                                      __nv_bfloat16* __restrict__ vt) {
  __shared__ __nv_bfloat16 tile[64][kTileN + 8];
  const int gb = blockIdx.x, n = blockIdx.y;
  for (int e = threadIdx.x; e < 64 * (kTileN / 8); e += blockDim.x) {
    const int p = e / (kTileN / 8), c8 = (e % (kTileN / 8)) * 8;
    const int d = n * kTileN + c8;
    const __nv_bfloat16* src = v + ((int64_t)gb * 64 + p) * D + d;
#pragma unroll
    for (int j = 0; j < 8; ++j) tile[p][c8 + j] = d + j < D ? src[j] : __float2bfloat16_rn(0.f);
  }
  __syncthreads();
  uint4* out = reinterpret_cast<uint4*>(vt + ((int64_t)n * NB + gb) * kTileN * 64);
  for (int e = threadIdx.x; e < kTileN * 8; e += blockDim.x) {
    const int r = e >> 3, p0 = (e & 7) * 8;
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __nv_bfloat162 b2 = __halves2bfloat162(tile[p0 + 2 * j][r], tile[p0 + 2 * j + 1][r]);
      w[j] = *reinterpret_cast<const uint32_t*>(&b2);
    }
    out[e] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// 64 x 64 blocked copy of a row-major weight [rows, cols] (BlockSparseLinear: rows = output features,
// cols = input features): tile (kb, j) holds rows [j*64, +64) x columns [kb*64, +64) as one contiguous
// 8 KB run at tile index kb * (rows / 64) + j, so the four column blocks of an output tile at one k-block
// are one 32 KB run when their blocks are consecutive, and one block is an 8 KB run otherwise (a
// row-major weight gives 64 pieces of 128 bytes, one per row, 8 KB apart at D_in = 4096).
__global__ void pack_blocked_kernel(const uint4* __restrict__ w, int64_t rows, int vec_per_row,
                                    uint4* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // over rows * vec_per_row 16-byte words
  if (i >= rows * vec_per_row) return;
  const int64_t nbo = rows / 64;
  const int c = (int)(i & 7);
  const int r = (int)((i >> 3) & 63);
  const int64_t t = i >> 9;  // tile = kb * nbo + j
  const int64_t kb = t / nbo, j = t - kb * nbo;
  out[i] = w[(j * 64 + r) * vec_per_row + kb * 8 + c];
}

// ============================================================================================
// Down projection: Y = H . V_sel + additive stream
// ============================================================================================
constexpr int kGroupM = 16;

__device__ __forceinline__ void down_tile(int tile, int m_tiles, int n_tiles, int& m, int& n) {
  const int per_group = kGroupM * n_tiles;
  const int group = tile / per_group;
  const int first_m = group * kGroupM;
  const int gsz = min(m_tiles - first_m, kGroupM);
  const int r = tile % per_group;
  m = first_m + r % gsz;
  n = r / gsz;
}

// Additive stream, bias and store of 32 consecutive computed columns [col0, col0 + 32) of one row per lane
// (the warp's lanes hold 32 rows).  `add`: add ctx16 . W_out^T and the bias (done by exactly one
// contributor of a tile).  With split-K (ks > 1) the fp32 partial of split `split` is stored instead of
// the output.  Computed column c lands in Y column omap[c / 64] * 64 + c % 64 (block-mapped form) or c;
// columns at or beyond `ncols` are not stored.
// The additive stream and the bias of one 32-column chunk (see down_store_chunk), in place.
__device__ __forceinline__ void down_add_chunk(const DownArgs& a, float (&o)[32], const float (&ctx)[16], int ocol0,
                                               bool add) {
  const int lane = threadIdx.x & 31;
  bool ctx_nz = false;  // rows without a context (another rank's tokens in a block shard) add nothing
#pragma unroll
  for (int k = 0; k < 16; ++k) ctx_nz |= ctx[k] != 0.f;
  if (a.ctx16 && add && __any_sync(0xffffffffu, ctx_nz)) {
    // o[i] += sum_k ctx[k] * W_out[ocol0 + i][k]; lane L loads row ocol0 + L of W_out and the warp
    // broadcasts it (all lanes of a chunk share the same 32 columns)
    float wv[16];
    const int64_t wrow = (int64_t)(ocol0 + lane) * 16;
    if (a.out_proj_f32) {
      const float4* wp = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.out_proj) + wrow);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float4 f = __ldg(wp + k);
        wv[4 * k] = f.x; wv[4 * k + 1] = f.y; wv[4 * k + 2] = f.z; wv[4 * k + 3] = f.w;
      }
    } else {
      const uint4* wp = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.out_proj) + wrow);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const uint4 u = __ldg(wp + k);
        const uint32_t ww[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          wv[8 * k + 2 * e] = __uint_as_float(ww[e] << 16);
          wv[8 * k + 2 * e + 1] = __uint_as_float(ww[e] & 0xFFFF0000u);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float sacc = 0.f;
#pragma unroll
      for (int k = 0; k < 16; ++k) sacc = fmaf(ctx[k], __shfl_sync(0xffffffffu, wv[k], i), sacc);
      o[i] += sacc;
    }
  }
  if (a.bias && add) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      o[i] += a.bias_f32 ? __ldg(reinterpret_cast<const float*>(a.bias) + ocol0 + i)
                         : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.bias)[ocol0 + i]);
  }
}

__device__ __forceinline__ void down_store_chunk(const DownArgs& a, float (&o)[32], const float (&ctx)[16],
                                                 int64_t row, bool row_ok, int col0, int ocol0, bool add, int split,
                                                 int ks, int ncols) {
  if (col0 >= ncols) return;  // uniform over the warp
  if (a.omap && (ocol0 < 0 || ocol0 + 32 > (a.ldy > 0 ? (int64_t)a.ldy : (int64_t)a.D))) {
    record_error(a.err, kErrBadTile);  // a block map entry outside Y: reported, nothing stored
    return;
  }
  down_add_chunk(a, o, ctx, ocol0, add);
  if (!row_ok) return;
  const int64_t ldy = a.ldy > 0 ? a.ldy : (int64_t)a.D;
  // output row: this rank's Y, or (peer output) the receive slot of the rank that owns the row
  void* ybase = a.y;
  int64_t yrow = row;
  if (a.peer_rows > 0 && ks == 1) {
    const int64_t owner = row / a.peer_rows;
    ybase = owner < kMaxPeers ? a.peer_y[owner] : nullptr;
    yrow = row - owner * a.peer_rows;
    if (!ybase) {
      record_error(a.err, kErrBadTile);  // a row past the ranks' slices: reported, not stored
      return;
    }
  }
  if (ks > 1) {  // partial of this split; summed in split order by a split-K reduce kernel
    float4* yp = reinterpret_cast<float4*>(a.y_acc + ((int64_t)split * a.M + row) * a.D + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) yp[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
  } else if (a.y_f32) {
    float4* yp = reinterpret_cast<float4*>(reinterpret_cast<float*>(ybase) + yrow * ldy + ocol0);
#pragma unroll
    for (int i = 0; i < 8; ++i) yp[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
  } else {
    uint4* yp = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(ybase) + yrow * ldy + ocol0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t pk[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 b2 = __floats2bfloat162_rn(o[8 * i + 2 * e], o[8 * i + 2 * e + 1]);
        pk[e] = *reinterpret_cast<const uint32_t*>(&b2);
      }
      yp[i] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  }
}

// Block-mapped form (DownArgs.nmap / omap / ncnt / kcnt): the B tile of a 256-column tile is loaded as
// four 64-row boxes from rows nmap[j]*64 (one box per column block j), tiles past the device count of
// column blocks are skipped by every role, and the k-loop runs over the device count of k-blocks (none:
// the tile's accumulator is taken as zero).
constexpr int kSmallDownStages = 0;  // 5: the small-batch variant below; 0: off

// S stages of AB bytes of H + 32 KB of V_t.  AB = 8 KB (batches of at most 64 tokens): the H box holds
// only the 64 rows that exist; the MMA still reads 128 rows, the upper 64 from the start of the stage's V_t
// tile, and the accumulator rows they produce (tokens >= M) are never stored.  The 8 KB saved per stage
// buy a fifth stage of V_t in flight.
template <int S, uint32_t AB>
__global__ void __launch_bounds__(kGemmThreads, 1)
down_kernel(const __grid_constant__ CUtensorMap tm_h, const __grid_constant__ CUtensorMap tm_vt,
            const __grid_constant__ CUtensorMap tm_vt_wide, const DownArgs a) {
  constexpr uint32_t kSB = AB + kBBytes;  // stage bytes
  using Bars = PipeBarsT<S>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = aligned_smem(smem_raw);
  Bars* bars = reinterpret_cast<Bars*>(smem + S * kSB);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tm_h);
    tma_prefetch_desc(&tm_vt);
  }
  pipe_init(bars, 4);
  griddep_wait();  // H (gate/up kernel) and the device counts are complete
  griddep_launch_dependents();
  const uint32_t tmem_base = bars->tmem;
  const int m_tiles = (int)((a.M + kTileM - 1) / kTileM);
  const int n_tiles = (a.D + kTileN - 1) / kTileN;
  const int ks = a.ksplit > 1 ? a.ksplit : 1;
  const int ntiles = m_tiles * n_tiles * ks;
  int nkb_all = a.K / kTileK;
  if (a.kcnt) nkb_all = max(0, min(nkb_all, *a.kcnt));
  int ncols = a.D;
  if (a.ncnt) ncols = max(0, min(a.D / kBlock, *a.ncnt)) * kBlock;
  uint32_t issued = 0;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        int m, n;
        down_tile(tile / ks, m_tiles, n_tiles, m, n);
        if (n * kTileN >= ncols) continue;
        const int sp = tile % ks;
        // split sp takes k-blocks sp, sp + ks, sp + 2 ks, ...: the splits of a tile read interleaved
        // pieces of the operands instead of one contiguous range each, which keeps their DRAM traffic
        // spread evenly over the memory (contiguous ranges per CTA measured up to 2x apart in time)
        const int kb0 = sp, kb1 = nkb_all;
        const int nv = a.nmap ? min(kTileN / kBlock, (ncols - n * kTileN) / kBlock) : 0;
        int nb[kTileN / kBlock];  // V_t row block of each valid column block, read once per tile
#pragma unroll
        for (int i = 0; i < kTileN / kBlock; ++i) nb[i] = i < nv ? a.nmap[n * (kTileN / kBlock) + i] : 0;
        // blocked weight with the tile's four column blocks consecutive: one 256-row (32 KB) box
        const bool wide4 = a.vt_blocked && nv == 4 && nb[1] == nb[0] + 1 && nb[2] == nb[0] + 2 && nb[3] == nb[0] + 3;
        const int nbo = a.D / kBlock;
        // H column block and parameter block of k-block j (touched-block list, pooled block map, or
        // strided identity), looked up one iteration ahead so that the load's latency overlaps the wait
        // for a free stage
        auto kmap = [&](int j) -> int2 {
          const int kh = a.ktiles ? a.ktiles[j].x % a.knbl : j;
          return make_int2(kh, a.bmap ? a.bmap[kh] : kh * a.stride + a.offset);
        };
        int2 kg_next = kb0 < kb1 ? kmap(kb0) : make_int2(0, 0);
        for (int kb = kb0; kb < kb1; kb += ks, ++it) {
          const int kh = kg_next.x, gb = kg_next.y;
          if (kb + ks < kb1) kg_next = kmap(kb + ks);
          const int s = it % S;
          const uint32_t ph = (it / S) & 1u;
          if (!mbar_wait(&bars->empty[s], ph ^ 1u, a.err, kErrWaitEmpty)) { ok = false; break; }
          uint8_t* As = smem + s * kSB;
          uint8_t* Bs = As + AB;
          if (a.nmap) {
            mbar_arrive_expect_tx(&bars->full[s], AB + (uint32_t)nv * (kBlock * kTileK * 2));
            tma_load_2d(As, &tm_h, &bars->full[s], kh * kTileK, m * kTileM);
            if (wide4) {
              tma_load_2d(Bs, &tm_vt_wide, &bars->full[s], 0, (gb * nbo + nb[0]) * kBlock);
            } else {
#pragma unroll
              for (int i = 0; i < kTileN / kBlock; ++i)
                if (i < nv) {
                  if (a.vt_blocked)
                    tma_load_2d(Bs + i * (kBlock * kTileK * 2), &tm_vt, &bars->full[s], 0, (gb * nbo + nb[i]) * kBlock);
                  else
                    tma_load_2d(Bs + i * (kBlock * kTileK * 2), &tm_vt, &bars->full[s], gb * kBlock, nb[i] * kBlock);
                }
            }
          } else {
            mbar_arrive_expect_tx(&bars->full[s], kSB);
            tma_load_2d(As, &tm_h, &bars->full[s], kh * kTileK, m * kTileM);
            if (a.vt_tiled)  // tile (n, gb) of the tile-contiguous V^T
              tma_load_2d(Bs, &tm_vt, &bars->full[s], 0, (n * (a.Np / kBlock) + gb) * kTileN);
            else
              tma_load_2d(Bs, &tm_vt, &bars->full[s], gb * kBlock, n * kTileN);
          }
        }
      }
      issued = it;
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      const uint32_t idesc = umma_idesc_bf16(kTileM, kTileN);
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        int m, n;
        down_tile(tile / ks, m_tiles, n_tiles, m, n);
        if (n * kTileN >= ncols) continue;
        const int sp = tile % ks;
        const int kb0 = sp, kb1 = nkb_all;  // interleaved k-blocks of split sp (see the producer)
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(&bars->acce[acc], aph ^ 1u, a.err, kErrWaitAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kTileN;
        for (int kb = kb0; kb < kb1; kb += ks) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1u;
          if (!mbar_wait(&bars->full[s], ph, a.err, kErrWaitFull)) { ok = false; break; }
          tc_fence_after();
          const uint64_t ad = umma_desc_sw128(smem_u32(smem + s * kSB));
          const uint64_t bd = umma_desc_sw128(smem_u32(smem + s * kSB + AB));
#pragma unroll
          for (int k = 0; k < kTileK / 16; ++k)
            umma_bf16(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
          umma_commit(&bars->empty[s]);
          ++it;
        }
        if (!ok) break;
        umma_commit(&bars->accf[acc]);
        ++local;
      }
      mma_quiesce(bars, it, a.err);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    int local = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      int m, n;
      down_tile(tile / ks, m_tiles, n_tiles, m, n);
      if (n * kTileN >= ncols) continue;
      const int split = tile % ks;
      const bool kempty = split >= nkb_all;  // interleaved k-blocks: split s has none when s >= nkb_all
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!warp_wait(&bars->accf[acc], aph, a.err, kErrWaitAccFull)) break;
      tc_fence_after();
      const int64_t row = (int64_t)m * kTileM + 32 * q + lane;
      const bool row_ok = row < a.M;
      // Y column of each of the tile's 4 column blocks (read once per tile)
      const int jb = n * (kTileN / kBlock);
      auto ocol_of = [&](int i) {
        return (a.omap && (jb + i) * kBlock < ncols) ? a.omap[jb + i] * kBlock : (jb + i) * kBlock;
      };
      const int ocb0 = ocol_of(0), ocb1 = ocol_of(1), ocb2 = ocol_of(2), ocb3 = ocol_of(3);
      float ctx[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) ctx[k] = 0.f;
      if (a.ctx16 && row_ok) {
        const float4* cp = reinterpret_cast<const float4*>(a.ctx16 + row * 16);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 f = __ldg(cp + i);
          ctx[4 * i] = f.x; ctx[4 * i + 1] = f.y; ctx[4 * i + 2] = f.z; ctx[4 * i + 3] = f.w;
        }
      }
      for (int c = 0; c < kTileN / 32; ++c) {
        uint32_t v[32];
        __syncwarp();
        tmem_ld32(tmem_base + acc * kTileN + c * 32 + ((uint32_t)(32 * q) << 16), v);
        tmem_ld_wait();
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = kempty ? 0.f : __uint_as_float(v[i]);
        const int col0 = n * kTileN + c * 32;
        // the additive stream and the bias of chunk c are added by split c % ks only: spread over the
        // splits (one split doing all of them made it the last to finish)
        down_store_chunk(a, o, ctx, row, row_ok, col0, ((c >> 1) == 0 ? ocb0 : (c >> 1) == 1 ? ocb1 : (c >> 1) == 2 ? ocb2 : ocb3) + (col0 & 63), c % ks == split, split, ks, ncols);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acce[acc]);
      ++local;
    }
  }
  if (a.peer_rows > 0) __threadfence_system();  // rows stored on other GPUs are visible there
  pipe_teardown(bars, issued, a.err);
}

// ============================================================================================
// Down projection on CTA pairs (cluster of 2, tcgen05 cta_group::2): a pair computes a 256-token x
// 256-column tile.  Each CTA loads its 128 rows of H and its 128 rows (output columns) of V_t per
// k-block (32 KB per stage instead of 48 KB for a 128 x 256 tile on one SM), the leader (even CTA)
// issues the pair MMAs, and each CTA drains its own 128 x 256 accumulator.  Six stages in flight.
// ============================================================================================
constexpr int kPairStages = 6;
constexpr uint32_t kPairABytes = kTileM * kTileK * 2;          // 16 KB: 128 rows of H
constexpr uint32_t kPairBBytes = (kTileN / 2) * kTileK * 2;    // 16 KB: 128 rows of V_t
constexpr uint32_t kPairStageBytes = kPairABytes + kPairBBytes;
using PairBars = PipeBarsT<kPairStages>;
// Peer output by TMA: per epilogue warp two 4 KB tiles (32 rows x 64 bf16 columns, 128-byte swizzle) in
// shared memory, stored to the owning rank while the warp fills the other one.
constexpr uint32_t kPeerTileBytes = 32 * 64 * 2;
constexpr uint32_t kPeerStageOffset = ((kPairStages * kPairStageBytes + sizeof(PairBars) + 1023) / 1024) * 1024;
constexpr size_t kPairSmem = 1024 + kPeerStageOffset + 4 * 2 * kPeerTileBytes;
static_assert(kPairSmem <= 227 * 1024, "pair down shared memory");
struct PeerMaps {
  CUtensorMap m[kMaxPeers];  // this rank's receive slot on rank o: [peer_rows, D] bf16, box 32 x 64
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
down2_kernel(const __grid_constant__ CUtensorMap tm_h, const __grid_constant__ CUtensorMap tm_vt,
             const __grid_constant__ CUtensorMap tm_vt_wide, const DownArgs a, const __grid_constant__ PeerMaps pm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = aligned_smem(smem_raw);
  PairBars* bars = reinterpret_cast<PairBars*>(smem + kPairStages * kPairStageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tm_h);
    tma_prefetch_desc(&tm_vt);
    if (a.nmap) tma_prefetch_desc(&tm_vt_wide);
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&bars->full[s], 1);   // leader: one expect_tx arrival + both CTAs' bytes
      mbar_init(&bars->empty[s], 1);  // arrival from the leader's commit
    }
    for (int c = 0; c < 2; ++c) {
      mbar_init(&bars->accf[c], 1);   // arrival from the leader's commit
      mbar_init(&bars->acce[c], 8);   // leader: the 4 epilogue warps of both CTAs
    }
    mbar_init(&bars->done, 1);
    bars->consumed = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc2(&bars->tmem, kTmemCols);
    tmem_relinquish2();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote arrival or pair commit
  tc_fence_after();
  griddep_wait();  // H (gate/up kernel) and the device counts are complete
  griddep_launch_dependents();
  const uint32_t tmem_base = bars->tmem;
  const int m_pairs = (int)((a.M + 2 * kTileM - 1) / (2 * kTileM));
  const int n_tiles = (a.D + kTileN - 1) / kTileN;
  const int tiles = m_pairs * n_tiles;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  // block-mapped form: both CTAs of a pair read the same device counts, so they skip the same tiles
  int nkb = a.K / kTileK;
  if (a.kcnt) nkb = max(0, min(nkb, *a.kcnt));
  int ncols = a.D;
  if (a.ncnt) ncols = max(0, min(a.D / kBlock, *a.ncnt)) * kBlock;
  constexpr uint32_t kBoxBytes = kBlock * kTileK * 2;  // one 64-row box of V_t
  uint32_t issued = 0;

  if (warp == 0) {
    // ---------------- producer (both CTAs): own rows of H, own half of the V_t tile (block-mapped form:
    // column blocks 2 * rank and 2 * rank + 1 of the tile, one 64-row box each)
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; tile < tiles && ok; tile += npairs) {
        int m, n;
        down_tile(tile, m_pairs, n_tiles, m, n);
        if (n * kTileN >= ncols) continue;
        const int nv = min(kTileN / kBlock, (ncols - n * kTileN) / kBlock);  // valid column blocks of the tile
        // this CTA's column blocks 2 * rank, 2 * rank + 1 of the tile: V_t row blocks, read once per tile
        const int j0 = n * (kTileN / kBlock) + 2 * (int)rank;
        const int mine = a.nmap ? max(0, min(2, nv - 2 * (int)rank)) : 0;
        const int b0 = mine > 0 ? a.nmap[j0] : 0;
        const int b1 = mine > 1 ? a.nmap[j0 + 1] : 0;
        const bool wide = mine == 2 && b1 == b0 + 1;  // consecutive blocks (the common case): one 128-row box
        const int nbo = a.D / kBlock;
        int gb_next = nkb > 0 ? (a.bmap ? a.bmap[0] : a.offset) : 0;  // one k-block ahead (see down_kernel)
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int gb = gb_next;
          if (kb + 1 < nkb) gb_next = a.bmap ? a.bmap[kb + 1] : (kb + 1) * a.stride + a.offset;
          const int s = it % kPairStages;
          const uint32_t ph = (it / kPairStages) & 1u;
          if (!mbar_wait(&bars->empty[s], ph ^ 1u, a.err, kErrWaitEmpty)) { ok = false; break; }
          uint8_t* As = smem + s * kPairStageBytes;
          uint8_t* Bs = As + kPairABytes;
          if (a.nmap) {
            if (leader) mbar_arrive_expect_tx(&bars->full[s], 2 * kPairABytes + (uint32_t)nv * kBoxBytes);
            tma_load_2d_pair(As, &tm_h, &bars->full[s], kb * kTileK, m * 2 * kTileM + (int)rank * kTileM);
            // row-major weight: box at (k column, weight row); blocked weight: tile rows (gb * nbo + block) * 64
            const int c0 = a.vt_blocked ? 0 : gb * kBlock;
            const int r0 = a.vt_blocked ? (gb * nbo + b0) * kBlock : b0 * kBlock;
            const int r1 = a.vt_blocked ? (gb * nbo + b1) * kBlock : b1 * kBlock;
            if (wide) {
              tma_load_2d_pair(Bs, &tm_vt_wide, &bars->full[s], c0, r0);
            } else {
              if (mine > 0) tma_load_2d_pair(Bs, &tm_vt, &bars->full[s], c0, r0);
              if (mine > 1) tma_load_2d_pair(Bs + kBoxBytes, &tm_vt, &bars->full[s], c0, r1);
            }
          } else {
            if (leader) mbar_arrive_expect_tx(&bars->full[s], 2 * kPairStageBytes);
            tma_load_2d_pair(As, &tm_h, &bars->full[s], kb * kTileK, m * 2 * kTileM + (int)rank * kTileM);
            if (a.vt_tiled)  // this CTA's half of tile (n, gb) of the tile-contiguous V^T
              tma_load_2d_pair(Bs, &tm_vt, &bars->full[s], 0,
                               (n * (a.Np / kBlock) + gb) * kTileN + (int)rank * (kTileN / 2));
            else
              tma_load_2d_pair(Bs, &tm_vt, &bars->full[s], gb * kBlock, n * kTileN + (int)rank * (kTileN / 2));
          }
        }
      }
      issued = it;
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- pair MMA issuer (leader only)
    if (leader && lane == 0) {
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      const uint32_t idesc = umma_idesc_bf16(2 * kTileM, kTileN);
      for (int tile = pair; tile < tiles && ok; tile += npairs) {
        int m, n;
        down_tile(tile, m_pairs, n_tiles, m, n);
        if (n * kTileN >= ncols) continue;
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait_cluster(&bars->acce[acc], aph ^ 1u, a.err, kErrWaitAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kTileN;
        for (int kb = 0; kb < nkb; ++kb) {
          const int s = it % kPairStages;
          const uint32_t ph = (it / kPairStages) & 1u;
          if (!mbar_wait_cluster(&bars->full[s], ph, a.err, kErrWaitFull)) { ok = false; break; }
          tc_fence_after();
          const uint64_t ad = umma_desc_sw128(smem_u32(smem + s * kPairStageBytes));
          const uint64_t bd = umma_desc_sw128(smem_u32(smem + s * kPairStageBytes + kPairABytes));
#pragma unroll
          for (int k = 0; k < kTileK / 16; ++k)
            umma2_bf16(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          umma2_commit(&bars->empty[s], 0x3);
          ++it;
        }
        if (!ok) break;
        umma2_commit(&bars->accf[acc], 0x3);
        ++local;
      }
      bars->consumed = (int32_t)it;
      umma2_commit(&bars->done, 0x1);
      if (!mbar_wait(&bars->done, 0, nullptr, 0)) record_error(a.err, kErrDrain);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (both CTAs): warp w drains TMEM lanes [32*(w%4), +32) of its CTA
    const int q = warp & 3;
    int local = 0;
    uint8_t* peer_stage = smem + kPeerStageOffset;
    uint32_t peer_buf = 0;
    for (int tile = pair; tile < tiles; tile += npairs) {
      int m, n;
      down_tile(tile, m_pairs, n_tiles, m, n);
      if (n * kTileN >= ncols) continue;
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!warp_wait(&bars->accf[acc], aph, a.err, kErrWaitAccFull)) break;
      tc_fence_after();
      const int64_t row = (int64_t)m * 2 * kTileM + (int64_t)rank * kTileM + 32 * q + lane;
      const bool row_ok = row < a.M;
      // Y column of each of the tile's 4 column blocks (read once per tile)
      const int jb = n * (kTileN / kBlock);
      auto ocol_of = [&](int i) {
        return (a.omap && (jb + i) * kBlock < ncols) ? a.omap[jb + i] * kBlock : (jb + i) * kBlock;
      };
      const int ocb0 = ocol_of(0), ocb1 = ocol_of(1), ocb2 = ocol_of(2), ocb3 = ocol_of(3);
      float ctx[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) ctx[k] = 0.f;
      if (a.ctx16 && row_ok) {
        const float4* cp = reinterpret_cast<const float4*>(a.ctx16 + row * 16);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 f = __ldg(cp + i);
          ctx[4 * i] = f.x; ctx[4 * i + 1] = f.y; ctx[4 * i + 2] = f.z; ctx[4 * i + 3] = f.w;
        }
      }
      const int64_t row0 = row - lane;  // the warp's first row
      if (a.peer_tma) {
        // peer output: 64-column pieces of the warp's 32 rows go to the owning rank by TMA from shared
        // memory (the stores run asynchronously; the warp only waits before refilling a tile buffer)
        const int owner = (int)(row0 / a.peer_rows);
        const bool store = row0 < a.M && owner < kMaxPeers;
        const int yrow0 = (int)(row0 - (int64_t)owner * a.peer_rows);
        for (int c2 = 0; c2 < kTileN / 64; ++c2) {
          uint8_t* tilebuf = peer_stage + (2 * q + (peer_buf & 1)) * kPeerTileBytes;
          if (lane == 0) bulk_wait_read<1>();  // this buffer's previous store has read it
          __syncwarp();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c = 2 * c2 + h;
            uint32_t v[32];
            __syncwarp();
            tmem_ld32(tmem_base + acc * kTileN + c * 32 + ((uint32_t)(32 * q) << 16), v);
            tmem_ld_wait();
            float o[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = nkb > 0 ? __uint_as_float(v[i]) : 0.f;
            const int col0 = n * kTileN + c * 32;
            down_add_chunk(a, o, ctx, col0, true);
            // row `lane` of the 128-byte swizzled tile: 16-byte piece j of the row at (j ^ lane % 8) * 16
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint32_t pk[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const __nv_bfloat162 b2 = __floats2bfloat162_rn(o[8 * j + 2 * e], o[8 * j + 2 * e + 1]);
                pk[e] = *reinterpret_cast<const uint32_t*>(&b2);
              }
              const int piece = 4 * h + j;
              *reinterpret_cast<uint4*>(tilebuf + lane * 128 + ((piece ^ (lane & 7)) << 4)) =
                  make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && store) {
            tma_store_2d(&pm.m[owner], smem_u32(tilebuf), n * kTileN + c2 * 64, yrow0);
            bulk_commit();
          }
          ++peer_buf;
        }
      } else {
        for (int c = 0; c < kTileN / 32; ++c) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld32(tmem_base + acc * kTileN + c * 32 + ((uint32_t)(32 * q) << 16), v);
          tmem_ld_wait();
          float o[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = nkb > 0 ? __uint_as_float(v[i]) : 0.f;  // no k-block: zero
          const int col0 = n * kTileN + c * 32;
          down_store_chunk(a, o, ctx, row, row_ok, col0, ((c >> 1) == 0 ? ocb0 : (c >> 1) == 1 ? ocb1 : (c >> 1) == 2 ? ocb2 : ocb3) + (col0 & 63), true, 0, 1, ncols);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_leader(&bars->acce[acc]);
      ++local;
    }
    if (a.peer_tma && lane == 0) bulk_wait_all();  // every peer store of this warp has completed
  }

  // ---------------- teardown: every MMA has completed (leader: done barrier; peer: its last accf), no
  // load of this CTA is in flight unless it aborted; then both CTAs free the pair's TMEM
  if (a.peer_rows > 0) __threadfence_system();  // rows stored on other GPUs are visible there
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && leader && aborted(a.err)) {
    for (uint32_t i = (uint32_t)bars->consumed; i < issued; ++i)
      if (!mbar_wait(&bars->full[i % kPairStages], (i / kPairStages) & 1u, nullptr, 0)) {
        record_error(a.err, kErrDrain);
        break;
      }
  }
  __syncthreads();
  cluster_sync();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc2(tmem_base, kTmemCols);
  }
}

// ============================================================================================
// Gate/up on CTA pairs for one active list shared by every token (pooled routing, the function-level
// Pattention, dense): a pair computes two parameter blocks x 256 tokens.  The even CTA's A operand is
// the 128 packed rows of block active[2p], the odd CTA's those of active[2p + 1]; each CTA loads 128 of
// the 256 token rows (TMA boxes of x), so both blocks share the token operand and one k-step moves
// 32 KB into each SM for 4.2 MFLOP (a one-SM 128 x 256 tile moves 48 KB).  Tiles run in groups of
// kGu2GroupP block pairs so that the concurrent tiles' weights and token rows stay in L2.  With an odd
// number of active blocks the last pair's odd CTA repeats the even CTA's block and stores nothing.
// ============================================================================================
constexpr int kGu2Stages = 6;
constexpr int kGu2GroupP = 8;
constexpr uint32_t kGu2ABytes = kTileM * kTileK * 2;  // 16 KB: 128 packed weight rows
constexpr uint32_t kGu2BBytes = kTileM * kTileK * 2;  // 16 KB: 128 token rows
constexpr uint32_t kGu2StageBytes = kGu2ABytes + kGu2BBytes;
using Gu2Bars = PipeBarsT<kGu2Stages>;
constexpr size_t kGu2Smem = 1024 + kGu2Stages * kGu2StageBytes + sizeof(Gu2Bars) + 64;
static_assert(kGu2Smem <= 227 * 1024, "pair gate/up shared memory");

__device__ __forceinline__ void gu2_tile(int tile, int P, int T, int& p, int& m) {
  const int per_group = kGu2GroupP * T;
  const int group = tile / per_group;
  const int first = group * kGu2GroupP;
  const int gsz = min(P - first, kGu2GroupP);
  const int r = tile % per_group;
  p = first + r % gsz;
  m = r / gsz;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
gateup2_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
               const GateUpArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = aligned_smem(smem_raw);
  Gu2Bars* bars = reinterpret_cast<Gu2Bars*>(smem + kGu2Stages * kGu2StageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
    for (int s = 0; s < kGu2Stages; ++s) {
      mbar_init(&bars->full[s], 1);   // leader: one expect_tx arrival + both CTAs' bytes
      mbar_init(&bars->empty[s], 1);  // arrival from the leader's commit
    }
    for (int c = 0; c < 2; ++c) {
      mbar_init(&bars->accf[c], 1);   // arrival from the leader's commit
      mbar_init(&bars->acce[c], 8);   // leader: the 4 epilogue warps of both CTAs
    }
    mbar_init(&bars->done, 1);
    bars->consumed = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc2(&bars->tmem, kTmemCols);
    tmem_relinquish2();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote arrival or pair commit
  tc_fence_after();
  griddep_wait();  // the active list and x are complete
  griddep_launch_dependents();
  const uint32_t tmem_base = bars->tmem;
  const int P = (a.n_keys + 1) / 2;
  const int T = (int)((a.M + 2 * kTileM - 1) / (2 * kTileM));
  const int tiles = P * T;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int nkb = a.D / kTileK;
  uint32_t issued = 0;

  // this CTA's key (slot of H) of pair p; the odd CTA of a lone last block repeats the even CTA's block
  auto my_key = [&](int p, bool& store) {
    const int key = 2 * p + (int)rank;
    store = key < a.n_keys;
    return store ? key : 2 * p;
  };

  if (warp == 0) {
    // ---------------- producer (both CTAs): own block's packed rows, own half of the token rows
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; tile < tiles && ok; tile += npairs) {
        int p, m;
        gu2_tile(tile, P, T, p, m);
        bool store;
        int b = a.active[my_key(p, store)];
        if (b < 0 || (int64_t)(b + 1) * kBlock > a.Np) {
          record_error(a.err, kErrBadTile);  // reported; the loads read block 0, the epilogue stores nothing
          b = 0;
        }
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kGu2Stages;
          const uint32_t ph = (it / kGu2Stages) & 1u;
          if (!mbar_wait(&bars->empty[s], ph ^ 1u, a.err, kErrWaitEmpty)) { ok = false; break; }
          uint8_t* As = smem + s * kGu2StageBytes;
          if (leader) mbar_arrive_expect_tx(&bars->full[s], 2 * kGu2StageBytes);
          tma_load_2d_pair(As, &tm_w, &bars->full[s], 0, (kb * (a.Np / kBlock) + b) * kTileM);
          tma_load_2d_pair(As + kGu2ABytes, &tm_x, &bars->full[s], kb * kTileK, m * 2 * kTileM + (int)rank * kTileM);
        }
      }
      issued = it;
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- pair MMA issuer (leader only)
    if (leader && lane == 0) {
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      const uint32_t idesc = umma_idesc_bf16(2 * kTileM, kTileN);
      for (int tile = pair; tile < tiles && ok; tile += npairs) {
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait_cluster(&bars->acce[acc], aph ^ 1u, a.err, kErrWaitAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kTileN;
        for (int kb = 0; kb < nkb; ++kb) {
          const int s = it % kGu2Stages;
          const uint32_t ph = (it / kGu2Stages) & 1u;
          if (!mbar_wait_cluster(&bars->full[s], ph, a.err, kErrWaitFull)) { ok = false; break; }
          tc_fence_after();
          const uint64_t ad = umma_desc_sw128(smem_u32(smem + s * kGu2StageBytes));
          const uint64_t bd = umma_desc_sw128(smem_u32(smem + s * kGu2StageBytes + kGu2ABytes));
#pragma unroll
          for (int k = 0; k < kTileK / 16; ++k)
            umma2_bf16(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          umma2_commit(&bars->empty[s], 0x3);
          ++it;
        }
        if (!ok) break;
        umma2_commit(&bars->accf[acc], 0x3);
        ++local;
      }
      bars->consumed = (int32_t)it;
      umma2_commit(&bars->done, 0x1);
      if (!mbar_wait(&bars->done, 0, nullptr, 0)) record_error(a.err, kErrDrain);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (both CTAs): this CTA's block over the pair's 256 tokens
    const int q = warp & 3;
    int local = 0;
    for (int tile = pair; tile < tiles; tile += npairs) {
      int p, m;
      gu2_tile(tile, P, T, p, m);
      bool store;
      const int key = my_key(p, store);
      const int b = a.active[key];
      store = store && b >= 0 && (int64_t)(b + 1) * kBlock <= a.Np;
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!warp_wait(&bars->accf[acc], aph, a.err, kErrWaitAccFull)) break;
      tc_fence_after();
      if (store) {
        for (int c = 0; c < kTileN / 32; ++c) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld32(tmem_base + acc * kTileN + c * 32 + ((uint32_t)(32 * q) << 16), v);
          tmem_ld_wait();
          const int64_t tok = (int64_t)m * 2 * kTileM + c * 32 + lane;
          gu_store_chunk(a, v, tok < a.M ? (int)tok : -1, key, q, lane);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_leader(&bars->acce[acc]);
      ++local;
    }
  }

  // ---------------- teardown (as in down2_kernel)
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && leader && aborted(a.err)) {
    for (uint32_t i = (uint32_t)bars->consumed; i < issued; ++i)
      if (!mbar_wait(&bars->full[i % kGu2Stages], (i / kGu2Stages) & 1u, nullptr, 0)) {
        record_error(a.err, kErrDrain);
        break;
      }
  }
  __syncthreads();
  cluster_sync();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc2(tmem_base, kTmemCols);
  }
}

// Sums the split-K partials [ks][n] in split order (deterministic) and writes the output dtype; 4 elements
// per thread (n % 4 == 0: D % 64 == 0 on the tensor-core path).
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int ks, int64_t n, void* out, int out_f32) {
  griddep_wait();  // every split's partial is stored
  const int64_t i = 4 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= n) return;
  store4(out, i, splitk_sum4(part, ks, n, i), out_f32);
}

// Block-mapped form: sums the split partials [ks][M][D] (computed columns) of the first 64 * ncnt
// columns in split order and stores column c of row m at Y column omap[c / 64] * 64 + c % 64 (or c).
__global__ void splitk_reduce_mapped_kernel(const float* __restrict__ part, int ks, int64_t M, int D,
                                            const int32_t* __restrict__ ncnt, const int32_t* __restrict__ omap,
                                            void* out, int64_t ldy, int out_f32) {
  griddep_wait();  // every split's partial is stored
  const int ncols = ncnt ? max(0, min(D / kBlock, *ncnt)) * kBlock : D;
  const int64_t n4 = M * ncols / 4;  // 4 consecutive columns per thread (ncols % 64 == 0)
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = 4 * i / ncols;
    const int c = (int)(4 * i - m * ncols);
    const float4 s = splitk_sum4(part, ks, M * (int64_t)D, m * D + c);
    const int64_t col = omap ? (int64_t)omap[c / kBlock] * kBlock + c % kBlock : c;
    if (col < 0 || col + 4 > ldy) continue;  // a block map entry outside Y (reported by the contraction)
    store4(out, m * ldy + col, s, out_f32);
  }
}

// ============================================================================================
// Host side
// ============================================================================================
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool encode_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                   uint32_t box_inner, uint32_t box_outer) {
  auto fn = get_encode();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static int set_smem(const void* fn) {
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem) == cudaSuccess
             ? FP_OK : FP_ERR_CUDA;
}

template <class Cfg>
static int launch_gateup_cfg(const GateUpArgs& a, cudaStream_t st) {
  CUtensorMap tx, tw;
  // w_gu in tile-contiguous form: rows of 64 elements, tile (b, kb) = rows [(kb * NB + b) * 128, +128)
  if (!encode_map_2d(&tx, a.x, a.D, a.M, (uint64_t)a.D * 2, kTileK, a.tiles ? 1 : Cfg::kN) ||
      !encode_map_2d(&tw, a.w_gu, kTileK, (uint64_t)a.Np * 2 * (a.D / kTileK), kTileK * 2, kTileK, kTileM))
    return FP_ERR_CUDA;
  static std::once_flag once;
  static int attr = FP_OK;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute((const void*)gateup_kernel<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)Cfg::kSmem) == cudaSuccess ? FP_OK : FP_ERR_CUDA;
  });
  if (attr != FP_OK) return attr;
  if (launch_pdl(gateup_kernel<Cfg>, dim3(a.num_sms), dim3(Cfg::kThreads), Cfg::kSmem, st, tx, tw, a) != cudaSuccess)
    return FP_ERR_CUDA;
  if (Cfg::kN == 64 && a.gu_ks > 1) {
    // the tile count is on the device: one CTA per possible tile, idle past it
    const int grid = std::max(1, std::min(a.max_tiles, a.num_sms * 4));
    if (launch_pdl(gateup_split_combine_kernel, dim3(grid), dim3(kGuCombineThreads), 0, st, a) != cudaSuccess)
      return FP_ERR_CUDA;
  }
  return FP_OK;
}

// Pair gate/up for a shared active list (see gateup2_kernel).
static int launch_gateup2(const GateUpArgs& a, cudaStream_t st) {
  CUtensorMap tx, tw;
  if (!encode_map_2d(&tx, a.x, a.D, a.M, (uint64_t)a.D * 2, kTileK, kTileM) ||
      !encode_map_2d(&tw, a.w_gu, kTileK, (uint64_t)a.Np * 2 * (a.D / kTileK), kTileK * 2, kTileK, kTileM))
    return FP_ERR_CUDA;
  static std::once_flag once;
  static int attr = FP_OK;
  static int max_pairs = 0;
  std::call_once(once, [&] {
    if (cudaFuncSetAttribute((const void*)gateup2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kGu2Smem) != cudaSuccess) {
      attr = FP_ERR_CUDA;
      return;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.num_sms & ~1);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = kGu2Smem;
    cudaLaunchAttribute cl;
    cl.id = cudaLaunchAttributeClusterDimension;
    cl.val.clusterDim.x = 2;
    cl.val.clusterDim.y = 1;
    cl.val.clusterDim.z = 1;
    cfg.attrs = &cl;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (const void*)gateup2_kernel, &cfg) != cudaSuccess) n = 0;
    max_pairs = n;
  });
  if (attr != FP_OK) return attr;
  if (max_pairs <= 0) return FP_ERR_CUDA;
  const int64_t tiles = (int64_t)((a.n_keys + 1) / 2) * ((a.M + 2 * kTileM - 1) / (2 * kTileM));
  if (tiles <= 0) return FP_OK;
  const int grid = 2 * (int)std::min<int64_t>(tiles, std::min(max_pairs, a.num_sms / 2));
  return launch_pdl(gateup2_kernel, dim3(grid), dim3(kGemmThreads), kGu2Smem, st, tx, tw, a) == cudaSuccess
             ? FP_OK : FP_ERR_CUDA;
}

int launch_gateup(const GateUpArgs& a, cudaStream_t st) {
  // the split of a tile's contraction: batches of at most 64 tokens with token lists, 16-aligned D split
  if (a.gu_ks > 1 && (!a.tiles || a.energy || a.M > GuSmall::kN || !a.gu_part || a.max_tiles < 1 ||
                      a.gu_ks > (a.D / kTileK)))
    return FP_ERR_INVALID_ARG;
  // a shared active list over more than 128 tokens: block pairs on CTA pairs
  if (!a.tiles && !a.energy && a.M > kTileM && a.num_sms >= 2) return launch_gateup2(a, st);
  // every tile of a batch of at most 64 tokens holds at most 64 tokens (a key's tokens are distinct)
  if (a.M <= GuSmall::kN) return launch_gateup_cfg<GuSmall>(a, st);
  return launch_gateup_cfg<GuBig>(a, st);
}

__global__ void energy_combine_kernel(const float* __restrict__ part, int64_t M, int NB, const float* __restrict__ vnorm,
                                      float* __restrict__ E) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // over M * NB
  if (i >= M * NB) return;
  const int64_t n = M * NB;
  const float s = ((part[i] + part[n + i]) + part[2 * n + i]) + part[3 * n + i];
  E[i] = s / 64.0f * vnorm[i % NB];
}

__global__ void iota_kernel(int32_t* out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = i;
}

int launch_energy_combine(const float* part, int64_t M, int NB, const float* vnorm, float* E, cudaStream_t st) {
  const int64_t n = M * NB;
  if (n <= 0) return FP_OK;
  energy_combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(part, M, NB, vnorm, E);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

int launch_iota(int32_t* out, int n, cudaStream_t st) {
  if (n <= 0) return FP_OK;
  iota_kernel<<<(n + 255) / 256, 256, 0, st>>>(out, n);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

int launch_pack_gate_up(const void* kg, const void* ku, int Np, int D, void* wgu, cudaStream_t st) {
  const int vec = D * 2 / 16;
  const int64_t n = 2LL * Np * vec;
  pack_gate_up_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>((const uint4*)kg, (const uint4*)ku, Np, vec,
                                                                    (uint4*)wgu);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

int launch_pack_blocked(const void* w, int rows, int cols, void* out, cudaStream_t st) {
  const int vec = cols / 8;
  const int64_t n = (int64_t)rows * vec;
  if (n <= 0) return FP_OK;
  pack_blocked_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>((const uint4*)w, rows, vec, (uint4*)out);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

int launch_pack_vt(const void* v, int Np, int D, void* vt, cudaStream_t st) {
  const int NB = Np / kBlock, ntiles = (D + kTileN - 1) / kTileN;
  if (ntiles > 65535) return FP_ERR_UNSUPPORTED;
  pack_vt_kernel<<<dim3((unsigned)NB, (unsigned)ntiles), 256, 0, st>>>((const __nv_bfloat16*)v, D, NB,
                                                                        (__nv_bfloat16*)vt);
  return cudaGetLastError() == cudaSuccess ? FP_OK : FP_ERR_CUDA;
}

int launch_down(const DownArgs& a, cudaStream_t st) {
  const bool mapped = a.nmap || a.omap || a.ncnt || a.kcnt || a.bias || a.ldy > 0;
  const int ks = a.ksplit > 1 ? a.ksplit : 1;
  // peer output: whole rows of the unmapped form, stored by the contraction itself (no split-K)
  if (a.peer_rows > 0 && (ks > 1 || a.omap || a.nmap || (a.ldy > 0 && a.ldy != a.D))) return FP_ERR_UNSUPPORTED;
  if (mapped && a.D % kBlock != 0) return FP_ERR_INVALID_ARG;
  if (a.vt_tiled && a.nmap) return FP_ERR_INVALID_ARG;
  if (a.vt_blocked && (!a.nmap || a.vt_tiled || a.Np % kBlock)) return FP_ERR_INVALID_ARG;
  if (a.ktiles && (!a.kcnt || a.knbl < 1 || a.bmap || a.M > kTileM)) return FP_ERR_INVALID_ARG;
  // tile-contiguous V^T: rows of 64 elements, ceil(D / 256) * (Np / 64) tiles of 256 rows
  const uint64_t vt_rows = (uint64_t)((a.D + kTileN - 1) / kTileN) * (a.Np / kBlock) * kTileN;
  // blocked weight: rows of 64 elements, (Np / 64) * (D / 64) tiles of 64 rows
  const uint64_t blk_rows = (uint64_t)(a.Np / kBlock) * (a.D / kBlock) * kBlock;
  CUtensorMap th, tv, tv4;
  if (!encode_map_2d(&th, a.h, a.K, a.M, (uint64_t)a.K * 2, kTileK, kTileM) ||
      !(a.vt_tiled ? encode_map_2d(&tv, a.v_t, kTileK, vt_rows, kTileK * 2, kTileK, kTileN)
        : a.vt_blocked ? encode_map_2d(&tv, a.v_t, kTileK, blk_rows, kTileK * 2, kTileK, kBlock)
                       : encode_map_2d(&tv, a.v_t, a.Np, a.D, (uint64_t)a.Np * 2, kTileK, a.nmap ? kBlock : kTileN)))
    return FP_ERR_CUDA;
  tv4 = tv;
  if (a.vt_blocked && !encode_map_2d(&tv4, a.v_t, kTileK, blk_rows, kTileK * 2, kTileK, kTileN)) return FP_ERR_CUDA;
  if (ks == 1 && a.M >= 2 * kTileM && a.num_sms >= 2) {
    // CTA pairs: 256 x 256 tiles, each CTA loading 128 rows of H and half of the V_t tile (two 64-row
    // boxes in the block-mapped form)
    CUtensorMap tv2, tvw;
    if (a.vt_tiled) {
      if (!encode_map_2d(&tv2, a.v_t, kTileK, vt_rows, kTileK * 2, kTileK, kTileN / 2)) return FP_ERR_CUDA;
      tvw = tv2;
    } else if (a.vt_blocked) {
      if (!encode_map_2d(&tv2, a.v_t, kTileK, blk_rows, kTileK * 2, kTileK, kBlock) ||
          !encode_map_2d(&tvw, a.v_t, kTileK, blk_rows, kTileK * 2, kTileK, 2 * kBlock))
        return FP_ERR_CUDA;
    } else if (!encode_map_2d(&tv2, a.v_t, a.Np, a.D, (uint64_t)a.Np * 2, kTileK, a.nmap ? kBlock : kTileN / 2) ||
               !encode_map_2d(&tvw, a.v_t, a.Np, a.D, (uint64_t)a.Np * 2, kTileK, kTileN / 2)) {
      return FP_ERR_CUDA;
    }
    static std::once_flag once2;
    static int attr2 = FP_OK;
    std::call_once(once2, [] {
      attr2 = cudaFuncSetAttribute((const void*)down2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)kPairSmem) == cudaSuccess ? FP_OK : FP_ERR_CUDA;
    });
    if (attr2 != FP_OK) return attr2;
    // pairs that can be resident at once (a pair needs two SMs of one GPC with ~200 KB free each)
    static std::once_flag once3;
    static int max_pairs = 0;
    std::call_once(once3, [&] {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(a.num_sms & ~1);
      cfg.blockDim = dim3(kGemmThreads);
      cfg.dynamicSmemBytes = kPairSmem;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = 2;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, (const void*)down2_kernel, &cfg) != cudaSuccess) n = 0;
      max_pairs = n;
    });
    if (max_pairs <= 0) return FP_ERR_CUDA;
    const int64_t ptiles = ((a.M + 2 * kTileM - 1) / (2 * kTileM)) * ((a.D + kTileN - 1) / kTileN);
    const int grid2 = 2 * (int)std::min<int64_t>(ptiles, std::min(max_pairs, a.num_sms / 2));
    // peer output of bf16 rows: the epilogue stores 32 x 64 tiles by TMA through one map per owning rank
    PeerMaps pm;
    std::memset(&pm, 0, sizeof(pm));
    DownArgs b = a;
    if (a.peer_rows > 0 && !a.y_f32 && a.peer_rows % 32 == 0 && a.peer_rows <= INT32_MAX) {
      bool ok = true;
      for (int o = 0; o < kMaxPeers && ok; ++o)
        if (a.peer_y[o])
          ok = encode_map_2d(&pm.m[o], a.peer_y[o], a.D, (uint64_t)a.peer_rows, (uint64_t)a.D * 2, 64, 32);
      if (!ok) return FP_ERR_CUDA;
      b.peer_tma = 1;
    }
    return launch_pdl(down2_kernel, dim3(grid2), dim3(kGemmThreads), kPairSmem, st, th, tv2, tvw, b, pm) == cudaSuccess
               ? FP_OK : FP_ERR_CUDA;
  }
  const int64_t tiles = ((a.M + kTileM - 1) / kTileM) * ((a.D + kTileN - 1) / kTileN) * ks;
  const int grid = (int)std::min<int64_t>(tiles, a.num_sms);
  if (grid <= 0) return FP_OK;
  if (ks > 1 && !a.y_acc) return FP_ERR_INVALID_ARG;
  if (kSmallDownStages > 0 && a.M <= kTileM / 2) {
    // at most 64 rows of H: 8 KB H boxes and five stages (measured 2 us slower than four 16 KB + 32 KB
    // stages at the decode shape, so not taken)
    constexpr int kS = 5;
    constexpr uint32_t kAB = kTileK * (kTileM / 2) * 2;
    constexpr size_t kSmem = 1024 + kS * (kAB + kBBytes) + sizeof(PipeBarsT<kS>) + 64;
    static_assert(kSmem <= 227 * 1024, "small down shared memory");
    static std::once_flag once_s;
    static int attr_s = FP_OK;
    std::call_once(once_s, [] {
      attr_s = cudaFuncSetAttribute((const void*)down_kernel<kS, kAB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kSmem) == cudaSuccess ? FP_OK : FP_ERR_CUDA;
    });
    if (attr_s != FP_OK) return attr_s;
    CUtensorMap th64;
    if (!encode_map_2d(&th64, a.h, a.K, a.M, (uint64_t)a.K * 2, kTileK, kTileM / 2)) return FP_ERR_CUDA;
    if (launch_pdl(down_kernel<kS, kAB>, dim3(grid), dim3(kGemmThreads), kSmem, st, th64, tv, tv4, a) != cudaSuccess)
      return FP_ERR_CUDA;
  } else {
    static std::once_flag once;
    static int attr = FP_OK;
    std::call_once(once, [] { attr = set_smem((const void*)down_kernel<kStages, kABytes>); });
    if (attr != FP_OK) return attr;
    if (launch_pdl(down_kernel<kStages, kABytes>, dim3(grid), dim3(kGemmThreads), kGemmSmem, st, th, tv, tv4, a) !=
        cudaSuccess)
      return FP_ERR_CUDA;
  }
  if (ks > 1 && mapped) {
    const int64_t n = a.M * (int64_t)a.D;
    const int rgrid = (int)std::max<int64_t>(1, std::min<int64_t>((n / 4 + 255) / 256, (int64_t)a.num_sms * 8));
    if (launch_pdl(splitk_reduce_mapped_kernel, dim3(rgrid), dim3(256), 0, st, (const float*)a.y_acc, ks, a.M, a.D,
                   a.ncnt, a.omap, a.y, a.ldy > 0 ? a.ldy : (int64_t)a.D, a.y_f32) != cudaSuccess)
      return FP_ERR_CUDA;
  } else if (ks > 1) {
    const int64_t n = a.M * (int64_t)a.D;
    if (launch_pdl(splitk_reduce_kernel, dim3((unsigned)((n / 4 + 255) / 256)), dim3(256), 0, st, (const float*)a.y_acc,
                   ks, n, a.y, a.y_f32) != cudaSuccess)
      return FP_ERR_CUDA;
  }
  return FP_OK;
}

int down_ksplit(int64_t M, int D, int nkb, int num_sms) {
  // Only batches whose output tiles fill at most half of the SMs are split: every split then streams the
  // same k-blocks of V_t at the same time as the other tiles (all CTAs move through the contraction in
  // step, so each V_t block is read from HBM once).  Shares of a tile that run at different k positions
  // (stream-K) were measured to re-read V_t from HBM several times at these shapes (V_t is 117 MB at 8B).
  const int64_t tiles = ((M + kTileM - 1) / kTileM) * ((D + kTileN - 1) / kTileN);
  if (tiles <= 0 || 2 * tiles > num_sms) return 1;
  int ks = (int)(num_sms / tiles);
  ks = std::min(ks, std::max(1, nkb / 4));  // at least 4 k-blocks per split
  return std::max(ks, 1);
}

}  // namespace fp
