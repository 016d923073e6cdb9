// Internal declarations shared by the CUDA translation units of libfovealpatt.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/foveal_pattention.h"
#include "fp_ptx.cuh"

namespace fp {

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

// Activation of the Pattention scores (pattention_triton.py:172-191 codes, :296-309 semantics): g = x.k_gate,
// u = x.k_up (used by SwiGLU only).  GELU is the erf form (F.gelu's default).  The tensor-core epilogue
// uses the fast exponential and division intrinsics (bf16 outputs); the CUDA-core path (fp32 models,
// 1e-4 tolerance) uses expf and an IEEE division.
template <bool kPrecise>
__device__ __forceinline__ float pattention_act(int act, float g, float u) {
  const float silu = kPrecise ? g / (1.0f + expf(-g)) : __fdividef(g, 1.0f + __expf(-g));
  switch (act) {
    case FP_ACT_SILU: return silu;
    case FP_ACT_GELU: return 0.5f * g * (1.0f + erff(g * 0.7071067811865476f));
    case FP_ACT_RELU: return fmaxf(g, 0.0f);
    case FP_ACT_RELU2: {
      const float r = fmaxf(g, 0.0f);
      return r * r;
    }
    default: return silu * u;  // FP_ACT_SWIGLU
  }
}

// Tile shapes of the tensor-core path.
constexpr int kTileM = 128;       // UMMA M: weight rows (gate/up) or tokens (down)
constexpr int kTileN = 256;       // UMMA N: tokens (gate/up) or output columns (down)
constexpr int kTileK = 64;        // one 128-byte swizzle row of bf16 = one parameter block
constexpr int kStages = 4;
constexpr int kBlock = 64;        // parameter tokens per block
constexpr int kGemmThreads = 192; // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
// gate/up kernel: at most kGuN tokens per tile (balanced tiles of a block's token list) and kGuStages
// pipeline stages of 16 KB (weights) + kGuN x 128 B (token rows) in shared memory
constexpr int kGuN = 256;
constexpr int kGuStages = 4;

// ---- router.cu
// k16f_cos (optional): fp32 block keys [NB, 16] of the cosine form (both sides L2-normalised,
// compute_block_scores core.py:254-266) used instead of k16.
int launch_router_scores(const void* x, const void* wq, const void* k16, int dtype, int64_t M, int D,
                         int NB, float temperature, float* scores, float* q16, cudaStream_t st,
                         const float* k16f_cos = nullptr);
struct SelectOut;
int launch_select(const float* scores, int64_t M, int NB, int base, float top_p, int k_min, int k_max,
                  int capacity, float temperature, int32_t* idx, int32_t* cnt, const float* k16f,
                  float* ctx16, float* stats, cudaStream_t st);
int launch_select_out(const float* scores, int64_t M, float temperature, const SelectOut& o, const float* k16f,
                      cudaStream_t st);
int launch_colmean(const void* a, int dtype, int64_t M, int D, float* part, float* mean, cudaStream_t st);
int launch_pooled_topk(const float* mean_vec, const void* wq, const void* k16, int dtype, int D, int NB,
                       int base, int remote, int mode, int32_t* active, float* mean_scores_out,
                       cudaStream_t st);

// Outputs and parameters of the per-token selection (select_blocks, core.py:46-160).
struct SelectOut {
  int NB, base;
  float top_p;
  int k_min, k_max, capacity;
  int32_t* idx;   // [M, capacity] sorted remote ids (nullptr: context-only mode)
  int32_t* cnt;   // [M]
  float* ctx16;   // optional [M, 16] additive-stream context softmax(S/T) . K16
  float* stats;   // optional [3]: capped tokens, sum of counts, base-only tokens
  int64_t ld = 0;     // row stride of the score matrix (0: NB)
  int id_offset = 0;  // added to every written block id
  int fast = 0;       // BlockSparseLinear's inference rule: count = min(#(cum < top_p) + 1, K_max), no
                      // clamp to the available blocks (block_matmul.py:190-193)
};

// Fused token routing (scores + selection + block CSR) of the token-routed forward.
// Block CSR: key = chunk(t) * nbl + slot(b) for the local blocks (b % stride == offset, slot = b / stride);
// each key owns a bucket of key_cap entries of pair_tok.  key_cnt and *ticket must be zero on entry.
// Runs of memory pulled into L2 while the routing kernels leave HBM idle (batches of at most 64 tokens):
// n runs of `bytes` starting at base + i * stride.
struct L2Prefetch {
  const char* base = nullptr;
  int64_t stride = 0, bytes = 0;
  int n = 0;
};

struct RouteArgs {
  const void* x;        // [M, D]
  const void* wq;       // [16, D]
  const void* k16;      // [NB, 16]
  int64_t M;
  int D, NB;
  float temperature;
  SelectOut sel;
  float* scores;        // optional [M, NB] router scores S (before the temperature)
  float* q16;           // optional [M, 16] normalised queries
  float* qraw;          // [M, 16] raw projections x W_q^T (workspace)
  uint4* hzero;         // optional: per-token rows of hrow_vec 16-byte words cleared (masked H)
  int64_t hrow_vec;
  int32_t* key_cnt;     // optional block CSR: [nkey] counters
  int32_t* pair_tok;    // [nkey * key_cap] token ids
  int64_t key_cap;
  int stride, offset, nbl, chunk, nkey;
  int2* tiles;          // gate/up work list: (key, first row) per tile
  int max_tiles;
  int32_t* meta;        // meta[0] = number of tiles, meta[1] = number of pairs
  unsigned int* ticket; // CTA completion counter
  int* err;
  int num_sms;
  // Given routes (block-sharded forward with the routing split over ranks): remote ids [M, given_cap]
  // and counts [M] computed elsewhere; the kernel then only builds the block lists, the tile list and the
  // H clears (no projection, scores or selection)
  const int32_t* given_idx = nullptr;
  const int32_t* given_cnt = nullptr;
  int given_cap = 0;
};
int launch_route(const RouteArgs& a, int dtype, cudaStream_t st);

// ---- gemm.cu (tensor-core path, bf16)
struct GateUpArgs {
  const void* x;        // [M, D] bf16
  const void* w_gu;     // 2 * Np * D bf16: packed gate/up rows, tile-contiguous (launch_pack_gate_up)
  int64_t M;
  int D, Np;
  // work list: explicit (tiles/meta from the routing kernel) or implicit (pooled: n_keys x ceil(M/256))
  const int2* tiles;
  const int32_t* meta;      // meta[0] = number of tiles (explicit mode)
  const int32_t* key_cnt;   // [nkey] tokens per key (explicit mode)
  const int32_t* pair_tok;  // token ids of key k at pair_tok[k * key_cap ...] (explicit mode)
  int64_t key_cap;
  int nbl, stride, offset;  // explicit mode: slot = key % nbl, block = slot * stride + offset
  const int32_t* active;    // implicit mode: block id of key j
  int n_keys;               // implicit mode: number of active blocks
  void* h;                  // [M, ldh] bf16 activations
  int64_t ldh;
  // energy mode (instead of writing h): energy[q][t][key] = sum over the 16 channels of TMEM quarter q of
  // |h[t, channel]| (fp32), for the teacher block energies of the offline calibration
  float* energy;
  int* err;
  int num_sms;
  int act = FP_ACT_SWIGLU;  // activation of the epilogue (non-gated forms ignore the up rows)
  // Split of each tile's contraction over D (batches of at most 64 tokens, explicit mode, no energy): work
  // unit u = (tile u / gu_ks, k-range u % gu_ks); each unit stores its fp32 accumulator to gu_part
  // [max_tiles][gu_ks][128][64], and a second kernel sums each tile's partials in split order and runs the
  // epilogue (activation, store into H).
  int gu_ks = 1;
  float* gu_part = nullptr;
  int max_tiles = 0;  // bound of the device tile count (sizes the second kernel's grid)
  // issued by every CTA before it waits for the routing kernel (batches of at most 64 tokens)
  L2Prefetch pf;
};
int launch_gateup(const GateUpArgs& a, cudaStream_t st);
// Work units of the decode split: k-blocks per unit at least 8, at most 4 units per tile.
__host__ __device__ __forceinline__ int gateup_decode_ksplit(int D) {
  const int nkb = D / 64;
  return nkb >= 32 ? 4 : (nkb >= 16 ? 2 : 1);
}
// E[t, b] = (sum_q part[q][t][b]) / 64 * vnorm[b], quarters summed in order
int launch_energy_combine(const float* part, int64_t M, int NB, const float* vnorm, float* E, cudaStream_t st);
int launch_iota(int32_t* out, int n, cudaStream_t st);
int launch_pack_gate_up(const void* kg, const void* ku, int Np, int D, void* wgu, cudaStream_t st);
// V^T tile-contiguous: ceil(D / 256) * (Np / 64) tiles of 256 x 64 (bf16), tile (n, b) at index n * NB + b.
int launch_pack_vt(const void* v, int Np, int D, void* vt, cudaStream_t st);
// 64 x 64 blocked copy of a row-major [rows, cols] bf16 matrix: tile (kb, j) = rows [j*64, +64) x columns
// [kb*64, +64), contiguous 8 KB at tile index kb * (rows / 64) + j.
int launch_pack_blocked(const void* w, int rows, int cols, void* out, cudaStream_t st);

// Rows per gate/up tile of a block-CSR key with `cnt` tokens: ceil(cnt / kGuN) tiles of equal size,
// rounded up to the UMMA N granularity (16).
__host__ __device__ __forceinline__ int balanced_rows(int cnt) {
  const int nt = (cnt + kGuN - 1) / kGuN;
  const int per = nt > 0 ? (cnt + nt - 1) / nt : 0;
  return (per + 15) & ~15;
}

// Peer-memory reduce-scatter (fp_peer.cu): ranks of one job, at most kMaxPeers.
constexpr int kMaxPeers = 8;
struct PeerFlags {
  uint32_t* flag[kMaxPeers];  // this rank's flag word on rank w (peer pointer; own rank: local)
  int world;
};
int launch_peer_signal(const PeerFlags& f, uint32_t epoch, cudaStream_t st);
// ---- api.cu
// Smallest workspace of the token forward (without the decode split's partials); the allocation-free entry
// point runs in it.
size_t token_workspace_size_min(int dtype, int64_t M, int D, int NB, int base_blocks, int max_remote,
                                int block_stride);

struct DownArgs {
  const void* h;        // [M, K] bf16
  const void* v_t;      // B operand: V^T tile-contiguous (vt_tiled, launch_pack_vt) or row-major [D, Np] bf16
  int64_t M;
  int D, Np, K;         // K = number of k-blocks * 64 read from h
  const int32_t* bmap;  // optional: global block of k-block j (pooled); else j*stride+offset
  int stride, offset;
  const float* ctx16;   // optional additive stream context [M, 16]
  const void* out_proj; // [D, 16] (bf16 or fp32 per out_proj_f32)
  int out_proj_f32;
  void* y;              // [M, D]
  int y_f32;
  int ksplit;           // > 1: split the k-blocks over CTAs; each split writes its fp32 partial
  float* y_acc;         // [ksplit, M, D] fp32 partials (ksplit > 1), summed in split order
  int* err;
  int num_sms;
  // Block-mapped form (one-SM kernel only; the union contractions of BlockSparseLinear and the
  // Tokenformer layer).  Output columns are handled in 64-wide column blocks j < D / 64:
  const int32_t* nmap = nullptr;  // B rows of column block j = v_t rows [nmap[j]*64, +64) (else j*64 + n)
  const int32_t* omap = nullptr;  // Y columns of column block j = [omap[j]*64, +64) (else [j*64, +64))
  const int32_t* ncnt = nullptr;  // device count of valid column blocks (else D / 64)
  const int32_t* kcnt = nullptr;  // device count of k-blocks (else K / 64)
  const void* bias = nullptr;     // optional per-Y-column bias (bf16, or fp32 per bias_f32)
  int bias_f32 = 0;
  int64_t ldy = 0;                // Y row stride in elements (0: D)
  int vt_tiled = 0;               // v_t in the tile-contiguous form of launch_pack_vt (the MLP's packed V)
  // k-block j of the contraction = H column block (and parameter block slot) ktiles[j].x % knbl, for j below
  // the device count kcnt: the routing kernel's gate/up tile list of a batch of at most 64 tokens (one tile
  // per touched block, in block order), so that only touched blocks are contracted
  const int2* ktiles = nullptr;
  int knbl = 1;
  int vt_blocked = 0;             // block-mapped form: v_t in the 64 x 64 blocked form of launch_pack_blocked
                                  // (tile of k-block kb and row block j at rows (kb * D/64 + j) * 64)
  // Peer output (parameter-block sharding): row r of Y goes to rank o = r / peer_rows, row r - o * peer_rows
  // of peer_y[o] (row stride D, dtype per y_f32; peer pointers through CUDA IPC) instead of to y.
  void* peer_y[kMaxPeers] = {};
  int64_t peer_rows = 0;
  int peer_tma = 0;  // set by launch_down: the pair kernel stores peer rows by TMA from shared memory
};
int launch_down(const DownArgs& a, cudaStream_t st);
// Split-K factor used by the down projection for M tokens (1 = none).  Small batches (decode) have too
// few output tiles to occupy the GPU, so the contraction over parameter blocks is split instead.
int down_ksplit(int64_t M, int D, int nkb, int num_sms);
constexpr int kMaxSms = 256;  // SM count assumed when the workspace is sized without a device to query

// ---- simt.cu (CUDA-core path: fp32 models and shapes the tensor-core path does not tile)
struct SimtArgs {
  const void* x;
  const void* k_gate;
  const void* k_up;
  const void* v;        // [Np, D] reference layout
  int dtype;
  int64_t M;
  int D, NB;
  // per-token lists (token mode) or a shared list (pooled mode)
  int base;
  const int32_t* ridx;  // [M, cap]
  const int32_t* rcnt;  // [M]
  int cap;
  const int32_t* active;
  int n_active;
  int stride, offset;   // local block filter (token mode)
  const float* ctx16;
  const void* out_proj;
  void* y;
  int y_f32;
  int D_out = 0;            // output width = v's columns (0: D)
  int act = FP_ACT_SWIGLU;  // activation; k_up may be null unless SwiGLU
};
int launch_simt(const SimtArgs& a, cudaStream_t st);

// ---- variants.cu (BlockSparseLinear / Tokenformer contractions over the union of selected blocks)
int launch_param_blocks_16d(const void* P, const void* wk, const void* wv, int dtype, int64_t N, int D,
                            float* kb, float* vb, cudaStream_t st);
int launch_union(const int32_t* idx, const int32_t* cnt, int64_t M, int capacity, int NB, int base,
                 int32_t* active, int32_t* n_active, cudaStream_t st);
int launch_rowact(const void* S, int s_bf16, int64_t lds, int64_t M, const int32_t* n_active, int mode, float div,
                  void* P, int64_t ldp, int p_f32, cudaStream_t st, int max_cols);
int launch_fill_inactive(const int32_t* blocks, const int32_t* n_active, int NB, int64_t M, const float* ctx16,
                         const void* out_proj, int dtype, void* out, int64_t ldo, int num_sms, cudaStream_t st);
int launch_transpose(const void* src, int64_t rows, int64_t cols, int dtype, void* dst, cudaStream_t st);
// CUDA-core contraction over mapped 64-wide blocks (see mapped_gemm_simt_kernel).
struct MappedGemm {
  const void* a; int64_t lda; int a_f32;
  const void* b; int64_t ldb; int b_f32;
  int nn;                 // 0: B rows are output columns (B[row(c), k]); 1: B rows are contraction indices
  int64_t M; int K, N;    // contraction length and computed columns (upper bounds)
  const int32_t* nmap; const int32_t* kmap; const int32_t* omap; const int32_t* ncnt; const int32_t* kcnt;
  const void* bias; int bias_f32;
  const float* ctx16; const void* out_proj; int out_proj_f32;
  void* y; int64_t ldy; int y_f32;
};
int launch_mapped_gemm_simt(const MappedGemm& g, cudaStream_t st);

// Launch `kern` with programmatic stream serialization (it may start during the previous kernel of the
// stream and must call griddep_wait() before reading that kernel's results).
template <typename... Exp, typename... Act>
inline cudaError_t launch_pdl(void (*kern)(Exp...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Act&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Act&&>(args)...);
}

// ---- tensor maps
bool encode_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                   uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer);

}  // namespace fp
