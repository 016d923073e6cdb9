// extern "C" entry points of libfovealpatt.so: argument validation, workspace layout and the launch
// sequence of each forward.  Declarations and contracts: include/foveal_pattention.h.
#include "fp_internal.cuh"

#include <algorithm>
#include <mutex>

namespace fp {
namespace {

constexpr size_t kAlign = 1024;

size_t align_up(size_t v, size_t a = kAlign) { return (v + a - 1) / a * a; }

struct Carve {
  size_t off = 0;
  size_t take(size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes);
    return o;
  }
};

// Token-chunk length of the block CSR: one chunk of x (bf16) is ~32 MB, so that the gate/up tiles of
// one chunk gather their token rows from L2.
int csr_chunk(int D) { return std::max(1024, (1 << 24) / std::max(D, 1)) / 128 * 128; }

int local_blocks(int NB, int stride, int offset) {
  return offset >= NB ? 0 : (NB - offset + stride - 1) / stride;
}

bool tensor_path(int dtype, int D) { return dtype == FP_DTYPE_BF16 && D % 64 == 0 && D >= 64; }

int layout_sms();

struct TokenLayout {
  size_t err, zero_bytes, key_cnt, meta, qraw, ridx, rcnt, ctx, pair_tok, tiles, h, yacc, gu_part, total;
  int ksplit, gu_ks;
  int nbl, chunk, nkey, max_tiles;
  int64_t key_cap;
};

constexpr size_t kTicketOffset = 128;  // CTA completion counter of the routing kernel, in the error area

// split: allow the decode split of the gate/up contraction (its fp32 partials need
// max_tiles * 4 * 32 KB); a workspace sized without it runs the unsplit kernel.
TokenLayout token_layout(int dtype, int64_t M, int D, int NB, int base, int kmax, int stride, int offset,
                         bool split = true) {
  TokenLayout L{};
  Carve c;
  L.nbl = local_blocks(NB, stride, offset);
  L.chunk = csr_chunk(D);
  const int64_t nchunks = (M + L.chunk - 1) / L.chunk;
  L.nkey = (int)(nchunks * std::max(L.nbl, 1));
  L.key_cap = std::min<int64_t>(L.chunk, std::max<int64_t>(M, 1));
  const bool tc = tensor_path(dtype, D);
  const int64_t pairs = M * (int64_t)(base + kmax);
  L.max_tiles = (int)(pairs / kGuN + L.nkey + 1);
  // batches of at most 64 tokens split each gate/up tile's contraction over D (work balance of the
  // decode step)
  L.gu_ks = split && tc && M <= 64 ? gateup_decode_ksplit(D) : 1;
  // error word, completion ticket and the block-CSR key counters: cleared by one memset per call.  The
  // error word stays at offset 0 (fp_noalloc_device_error reads it there in the library's scratch array).
  L.zero_bytes = 256 + (tc ? (size_t)L.nkey * 4 : 0);
  L.err = c.take(L.zero_bytes);
  L.key_cnt = L.err + 256;
  L.meta = c.take(64);
  L.qraw = c.take((size_t)M * 16 * 4);
  L.ridx = c.take((size_t)M * std::max(kmax, 1) * 4);
  L.rcnt = c.take((size_t)M * 4);
  L.ctx = c.take((size_t)M * 16 * 4);
  if (tc) {
    L.pair_tok = c.take((size_t)L.nkey * L.key_cap * 4);
    L.tiles = c.take((size_t)L.max_tiles * 8);
    L.h = c.take((size_t)M * L.nbl * kBlock * 2);
    L.ksplit = down_ksplit(M, D, std::max(L.nbl, 1), layout_sms());
    if (L.ksplit > 1) L.yacc = c.take((size_t)L.ksplit * M * D * 4);
    if (L.gu_ks > 1) L.gu_part = c.take((size_t)L.max_tiles * L.gu_ks * kTileM * 64 * 4);
  }
  L.total = c.off;
  return L;
}

struct PooledLayout {
  size_t err, part, mean, h, yacc, total;
  int ksplit;
};

PooledLayout pooled_layout(int dtype, int64_t M, int D, int NB, int n_active) {
  PooledLayout L{};
  Carve c;
  L.err = c.take(256);
  const int64_t nchunk = (M + 255) / 256;
  const int width = std::max(D, NB);
  L.part = c.take((size_t)nchunk * width * 4);
  L.mean = c.take((size_t)width * 4);
  if (tensor_path(dtype, D)) {
    L.h = c.take((size_t)M * std::max(n_active, 1) * kBlock * 2);
    L.ksplit = down_ksplit(M, D, std::max(n_active, 1), layout_sms());
    if (L.ksplit > 1) L.yacc = c.take((size_t)L.ksplit * M * D * 4);
  }
  L.total = c.off;
  return L;
}

template <typename T>
T* at(void* ws, size_t off) { return reinterpret_cast<T*>(reinterpret_cast<char*>(ws) + off); }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Every launching entry point starts here.  Launch checks read the runtime's per-thread last error, so a
// non-sticky error left by earlier, unrelated calls of the caller's thread is cleared first (a sticky
// error, such as a fault of the context, still fails every launch).
int device_info(int& num_sms) {
  (void)cudaGetLastError();
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FP_ERR_CUDA;
  static int cache_sms[64] = {0};
  static int cache_major[64] = {0};
  if (dev < 64 && cache_sms[dev] > 0) {
    num_sms = cache_sms[dev];
    return cache_major[dev] == 10 ? FP_OK : FP_ERR_DEVICE;
  }
  int major = 0, sms = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return FP_ERR_CUDA;
  if (dev < 64) {
    cache_sms[dev] = sms;
    cache_major[dev] = major;
  }
  num_sms = sms;
  return major == 10 ? FP_OK : FP_ERR_DEVICE;
}

// SM count the split-K choice of the workspace layout is made for; kMaxSms when no device can be queried
// (a layout for more splits is never smaller).
int layout_sms() {
  int sms = 0;
  if (device_info(sms) == FP_OK && sms > 0 && sms <= kMaxSms) return sms;
  return kMaxSms;
}

int check_common(int dtype, int64_t M, int D, int NB) {
  if (dtype != FP_DTYPE_F32 && dtype != FP_DTYPE_BF16) return FP_ERR_UNSUPPORTED;
  if (M < 0 || D <= 0 || NB <= 0) return FP_ERR_INVALID_ARG;
  if (D % 8 != 0 || NB > 1024) return FP_ERR_UNSUPPORTED;
  if (M > (int64_t)INT32_MAX / 8) return FP_ERR_UNSUPPORTED;
  return FP_OK;
}

thread_local cudaEvent_t g_stage_events[8];
thread_local int g_n_stage = 0;

inline void stage_mark(int i, cudaStream_t st) {
  if (i < g_n_stage && g_stage_events[i]) cudaEventRecord(g_stage_events[i], st);
}

#define FP_TRY(expr)              \
  do {                            \
    const int _s = (expr);        \
    if (_s != FP_OK) return _s;   \
  } while (0)

}  // namespace

// The smallest workspace the token forward accepts (without the decode split's partials).
size_t token_workspace_size_min(int dtype, int64_t M, int D, int NB, int base_blocks, int max_remote,
                                int block_stride) {
  return token_layout(dtype, M, D, NB, base_blocks, max_remote, std::max(block_stride, 1), 0, false).total;
}
}  // namespace fp

using namespace fp;

extern "C" {

int fp_abi_version(void) { return FP_ABI_VERSION; }

const char* fp_status_string(int status) {
  switch (status) {
    case FP_OK: return "ok";
    case FP_ERR_INVALID_ARG: return "invalid argument (null pointer, shape, parameter or alignment)";
    case FP_ERR_UNSUPPORTED: return "unsupported dtype or shape";
    case FP_ERR_WORKSPACE: return "workspace too small";
    case FP_ERR_CUDA: return "CUDA runtime error or launch failure";
    case FP_ERR_DEVICE: return "current device is not an sm_100 GPU";
    case FP_ERR_TIMEOUT: return "a kernel's bounded wait ran out";
    default: return "unknown status";
  }
}

int fp_router_scores(const void* x, const void* q_proj, const void* block_keys, int dtype, int64_t M, int D,
                     int NB, float* scores, float* q16, void* stream) {
  FP_TRY(check_common(dtype, M, D, NB));
  if (!x || !q_proj || !block_keys || !scores) return FP_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(q_proj)) return FP_ERR_INVALID_ARG;
  int sms;
  FP_TRY(device_info(sms));
  return launch_router_scores(x, q_proj, block_keys, dtype, M, D, NB, 1.0f, scores, q16,
                              (cudaStream_t)stream);
}

int fp_select_blocks(const float* scores, int64_t M, int NB, int base_blocks, float top_p, int min_remote,
                     int max_remote, int capacity, float temperature, int32_t* remote_indices,
                     int32_t* remote_counts, const float* block_keys_f32, float* ctx16, float* stats,
                     void* stream) {
  if (M < 0 || NB <= 0 || NB > 1024 || base_blocks < 0 || capacity < 0 || min_remote < 0 || max_remote < 0)
    return FP_ERR_INVALID_ARG;
  if (!scores || !(temperature > 0.f)) return FP_ERR_INVALID_ARG;
  if ((block_keys_f32 == nullptr) != (ctx16 == nullptr)) return FP_ERR_INVALID_ARG;
  if (remote_indices == nullptr && ctx16 == nullptr) return FP_ERR_INVALID_ARG;
  if (remote_indices && (!remote_counts || capacity <= 0)) return FP_ERR_INVALID_ARG;
  int sms;
  FP_TRY(device_info(sms));
  return launch_select(scores, M, NB, base_blocks, top_p, min_remote, max_remote, capacity, temperature,
                       remote_indices, remote_counts, block_keys_f32, ctx16, stats, (cudaStream_t)stream);
}

size_t fp_pooled_workspace_size(int dtype, int64_t M, int D, int NB, int n_active) {
  return pooled_layout(dtype, M, D, NB, n_active).total;
}

size_t fp_token_workspace_size(int dtype, int64_t M, int D, int NB, int base_blocks, int max_remote,
                               int block_stride) {
  return token_layout(dtype, M, D, NB, base_blocks, max_remote, std::max(block_stride, 1), 0).total;
}


int fp_pooled_route(const void* x, const void* q_proj, const void* block_keys, int dtype, int64_t M, int D,
                    int NB, int base_blocks, int remote_blocks, int mode, const float* token_scores,
                    int32_t* active, float* mean_scores, void* workspace, size_t workspace_bytes,
                    void* stream) {
  FP_TRY(check_common(dtype, M, D, NB));
  if (!q_proj || !block_keys || !active || !workspace || M <= 0) return FP_ERR_INVALID_ARG;
  if (base_blocks < 0 || remote_blocks < 0 || base_blocks + remote_blocks > NB) return FP_ERR_INVALID_ARG;
  if (NB > 4096) return FP_ERR_UNSUPPORTED;
  if (mode == 0 && !x) return FP_ERR_INVALID_ARG;
  if (mode == 1 && !token_scores) return FP_ERR_INVALID_ARG;
  if (mode != 0 && mode != 1) return FP_ERR_INVALID_ARG;
  const PooledLayout L = pooled_layout(dtype, M, D, NB, 0);
  if (workspace_bytes < L.total) return FP_ERR_WORKSPACE;
  int sms;
  FP_TRY(device_info(sms));
  cudaStream_t st = (cudaStream_t)stream;
  float* part = at<float>(workspace, L.part);
  float* mean = at<float>(workspace, L.mean);
  if (mode == 0) FP_TRY(launch_colmean(x, dtype, M, D, part, mean, st));
  else FP_TRY(launch_colmean(token_scores, FP_DTYPE_F32, M, NB, part, mean, st));
  return launch_pooled_topk(mean, q_proj, block_keys, dtype, D, NB, base_blocks, remote_blocks, mode, active,
                            mean_scores, st);
}

int fp_pack_weights(const void* k_gate, const void* k_up, const void* v, int dtype, int Np, int D, void* w_gu,
                    void* v_t, void* stream) {
  if (!k_gate || !k_up || !v || !w_gu || !v_t || Np <= 0 || D <= 0) return FP_ERR_INVALID_ARG;
  if (dtype != FP_DTYPE_BF16) return FP_ERR_UNSUPPORTED;
  if (Np % kBlock || D % 64) return FP_ERR_UNSUPPORTED;
  if (!aligned16(k_gate) || !aligned16(k_up) || !aligned16(w_gu)) return FP_ERR_INVALID_ARG;
  int sms;
  FP_TRY(device_info(sms));
  cudaStream_t st = (cudaStream_t)stream;
  FP_TRY(launch_pack_gate_up(k_gate, k_up, Np, D, w_gu, st));
  return launch_pack_vt(v, Np, D, v_t, st);
}

int fp_pattention_token_fwd(const void* x, int64_t M, int D, int NB, int dtype, const void* k_gate,
                            const void* k_up, const void* v, const void* w_gu, const void* v_t, const void* q_proj,
                            const void* block_keys, const void* out_proj, int base_blocks, float top_p,
                            int min_remote, int max_remote, float temperature, int additive,
                            int block_stride, int block_offset, void* y, int y_f32,
                            int32_t* remote_indices, int32_t* remote_counts, float* scores,
                            void* workspace, size_t workspace_bytes, void* stream) {
  FP_TRY(check_common(dtype, M, D, NB));
  if (M == 0) return FP_OK;  // empty batch: nothing to do (empty tensors may carry null pointers)
  if (!x || !k_gate || !k_up || !v || !q_proj || !block_keys || !y || !workspace) return FP_ERR_INVALID_ARG;
  if (additive && !out_proj) return FP_ERR_INVALID_ARG;
  if (base_blocks < 0 || base_blocks > NB || min_remote < 0 || max_remote < 0) return FP_ERR_INVALID_ARG;
  if (block_stride < 1 || block_offset < 0 || block_offset >= block_stride) return FP_ERR_INVALID_ARG;
  if (!(temperature > 0.f)) return FP_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(q_proj)) return FP_ERR_INVALID_ARG;
  const bool tc = tensor_path(dtype, D);
  if (tc && (!v_t || !w_gu || !aligned16(v_t) || !aligned16(w_gu))) return FP_ERR_INVALID_ARG;
  if (!tc && D > 32 * 256) return FP_ERR_UNSUPPORTED;
  const int cap = std::max(max_remote, 1);
  TokenLayout L = token_layout(dtype, M, D, NB, base_blocks, max_remote, block_stride, block_offset);
  if (workspace_bytes < L.total)  // a smaller workspace (the no-alloc scratch): no decode split
    L = token_layout(dtype, M, D, NB, base_blocks, max_remote, block_stride, block_offset, false);
  if (workspace_bytes < L.total) return FP_ERR_WORKSPACE;
  int sms;
  FP_TRY(device_info(sms));
  cudaStream_t st = (cudaStream_t)stream;
  int* err = at<int>(workspace, L.err);
  if (cudaMemsetAsync(err, 0, L.zero_bytes, st) != cudaSuccess) return FP_ERR_CUDA;

  int32_t* ridx = remote_indices ? remote_indices : at<int32_t>(workspace, L.ridx);
  int32_t* rcnt = remote_counts ? remote_counts : at<int32_t>(workspace, L.rcnt);
  float* ctx = additive ? at<float>(workspace, L.ctx) : nullptr;
  const int nbl = L.nbl;
  const bool csr = tc && nbl > 0;

  stage_mark(0, st);
  // scores, selection and (tensor-core path) the block-major token lists in one kernel; the masked
  // activations H must read zero for unselected (token, block) pairs, so the routing warps clear each
  // token's row of H while they work (HBM is otherwise idle there)
  RouteArgs r{};
  r.x = x; r.wq = q_proj; r.k16 = block_keys; r.M = M; r.D = D; r.NB = NB; r.temperature = temperature;
  r.sel = SelectOut{NB, base_blocks, top_p, min_remote, max_remote, cap, ridx, rcnt, ctx, nullptr};
  r.scores = scores; r.q16 = nullptr; r.qraw = at<float>(workspace, L.qraw); r.err = err; r.num_sms = sms;
  int32_t* key_cnt = at<int32_t>(workspace, L.key_cnt);
  int32_t* pair_tok = csr ? at<int32_t>(workspace, L.pair_tok) : nullptr;
  int2* tiles = csr ? at<int2>(workspace, L.tiles) : nullptr;
  int32_t* meta = at<int32_t>(workspace, L.meta);
  void* h = csr ? at<void>(workspace, L.h) : nullptr;
  if (csr) {
    r.hzero = static_cast<uint4*>(h); r.hrow_vec = (int64_t)nbl * kBlock * 2 / 16;
    r.key_cnt = key_cnt; r.pair_tok = pair_tok; r.key_cap = L.key_cap;
    r.stride = block_stride; r.offset = block_offset; r.nbl = nbl; r.chunk = L.chunk; r.nkey = L.nkey;
    r.tiles = tiles; r.max_tiles = L.max_tiles; r.meta = meta;
    r.ticket = reinterpret_cast<unsigned int*>(at<char>(workspace, L.err + kTicketOffset));
  }
  FP_TRY(launch_route(r, dtype, st));
  stage_mark(1, st);

  if (!csr) {
    // CUDA-core path; a shard that owns no block contributes only the additive stream (or zeros).
    SimtArgs a{};
    a.x = x; a.k_gate = k_gate; a.k_up = k_up; a.v = v; a.dtype = dtype; a.M = M; a.D = D; a.NB = NB;
    a.base = base_blocks; a.ridx = ridx; a.rcnt = rcnt; a.cap = cap;
    a.active = L.nbl == 0 ? ridx : nullptr; a.n_active = 0;
    a.stride = block_stride; a.offset = block_offset; a.ctx16 = ctx; a.out_proj = out_proj; a.y = y;
    a.y_f32 = y_f32;
    return launch_simt(a, st);
  }
  stage_mark(2, st);
  GateUpArgs g{};
  g.x = x; g.w_gu = w_gu; g.M = M; g.D = D; g.Np = NB * kBlock;
  g.tiles = tiles; g.meta = meta; g.key_cnt = key_cnt; g.pair_tok = pair_tok; g.key_cap = L.key_cap;
  g.nbl = nbl; g.stride = block_stride; g.offset = block_offset; g.active = nullptr; g.n_keys = 0;
  g.h = h; g.ldh = (int64_t)nbl * kBlock; g.err = err; g.num_sms = sms;
  if (L.gu_ks > 1) {
    g.gu_ks = L.gu_ks; g.gu_part = at<float>(workspace, L.gu_part); g.max_tiles = L.max_tiles;
  }
  if (M <= 64 && block_stride == 1) {
    // HBM is idle while the routing kernels run, and the gate/up CTAs start (programmatic launch) on the
    // SMs the routing leaves free: each pulls a share of the packed gate/up tiles of the lowest block ids
    // (the first work units take the touched blocks in ascending order) into L2, about half of L2 (96 MB
    // measured slower)
    const int64_t tile_bytes = (int64_t)kTileM * kTileK * 2;  // 16 KB: one block at one k-block
    const int nkb = D / kTileK;
    const int64_t budget = 64ll << 20;
    const int nblk = (int)std::min<int64_t>(NB, budget / ((int64_t)nkb * tile_bytes));
    if (nblk > 0) {
      g.pf.base = static_cast<const char*>(w_gu);
      g.pf.stride = (int64_t)NB * tile_bytes;  // tile (kb, b) at (kb * NB + b) * 16 KB
      g.pf.bytes = (int64_t)nblk * tile_bytes;
      g.pf.n = nkb;
    }
  }
  FP_TRY(launch_gateup(g, st));
  stage_mark(3, st);
  DownArgs d{};
  d.h = h; d.v_t = v_t; d.vt_tiled = 1; d.M = M; d.D = D; d.Np = NB * kBlock; d.K = nbl * kBlock; d.bmap = nullptr;
  d.stride = block_stride; d.offset = block_offset; d.ctx16 = ctx; d.out_proj = out_proj;
  d.out_proj_f32 = dtype == FP_DTYPE_F32; d.y = y; d.y_f32 = y_f32; d.err = err; d.num_sms = sms;
  d.ksplit = L.ksplit; d.y_acc = L.ksplit > 1 ? at<float>(workspace, L.yacc) : nullptr;
  if (M <= 64) {
    // one gate/up tile per touched block, in block order: contract over the touched blocks only
    d.ktiles = tiles; d.knbl = nbl; d.kcnt = meta;
  }
  FP_TRY(launch_down(d, st));
  stage_mark(4, st);
  return FP_OK;
}

size_t fp_route_workspace_size(int64_t M) {
  Carve c;
  c.take(256);                                            // error word
  c.take((size_t)std::max<int64_t>(M, 0) * 16 * 4);       // raw 16-D queries
  return c.off;
}

int fp_route_tokens(const void* x, int64_t M, int D, int NB, int dtype, const void* q_proj, const void* block_keys,
                    int base_blocks, float top_p, int min_remote, int max_remote, float temperature,
                    int32_t* remote_indices, int32_t* remote_counts, float* ctx16, float* scores, void* workspace,
                    size_t workspace_bytes, void* stream) {
  FP_TRY(check_common(dtype, M, D, NB));
  if (M == 0) return FP_OK;
  if (!x || !q_proj || !block_keys || !remote_indices || !remote_counts || !workspace) return FP_ERR_INVALID_ARG;
  if (base_blocks < 0 || base_blocks > NB || min_remote < 0 || max_remote < 0) return FP_ERR_INVALID_ARG;
  if (!(temperature > 0.f)) return FP_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(q_proj)) return FP_ERR_INVALID_ARG;
  if (workspace_bytes < fp_route_workspace_size(M)) return FP_ERR_WORKSPACE;
  int sms;
  FP_TRY(device_info(sms));
  cudaStream_t st = (cudaStream_t)stream;
  int* err = at<int>(workspace, 0);
  if (cudaMemsetAsync(err, 0, 256, st) != cudaSuccess) return FP_ERR_CUDA;
  RouteArgs r{};
  r.x = x; r.wq = q_proj; r.k16 = block_keys; r.M = M; r.D = D; r.NB = NB; r.temperature = temperature;
  r.sel = SelectOut{NB, base_blocks, top_p, min_remote, max_remote, std::max(max_remote, 1), remote_indices,
                    remote_counts, ctx16, nullptr};
  r.scores = scores; r.q16 = nullptr; r.qraw = at<float>(workspace, 256); r.err = err; r.num_sms = sms;
  return launch_route(r, dtype, st);
}

namespace {
// Peer output of the routed forward: partial rows to the ranks that own them, then the writer's flag.
struct PeerSpec {
  void* const* out;        // [world] this rank's receive slot on each rank
  uint32_t* const* flags;  // [world] this rank's flag word on each rank
  int world;
  int64_t rows;            // token rows per rank
  uint32_t epoch;
};

int routed_fwd_impl(const void* x, int64_t M, int D, int NB, int dtype, const void* k_gate, const void* k_up,
                    const void* v, const void* w_gu, const void* v_t, const void* out_proj, int base_blocks,
                    int capacity, const int32_t* remote_indices, const int32_t* remote_counts, const float* ctx16,
                    int block_stride, int block_offset, void* y, int y_f32, void* workspace, size_t workspace_bytes,
                    void* stream, const PeerSpec* peer) {
  FP_TRY(check_common(dtype, M, D, NB));
  if (M == 0) return FP_OK;
  if (!x || !k_gate || !k_up || !v || (!y && !peer) || !workspace || !remote_counts) return FP_ERR_INVALID_ARG;
  if (peer) {
    if (peer->world < 1 || peer->world > kMaxPeers || !peer->out || !peer->flags || peer->rows <= 0 ||
        M != (int64_t)peer->world * peer->rows)
      return FP_ERR_INVALID_ARG;
    for (int w = 0; w < peer->world; ++w)
      if (!peer->out[w] || !peer->flags[w] || !aligned16(peer->out[w])) return FP_ERR_INVALID_ARG;
  }
  if (capacity < 0 || (capacity > 0 && !remote_indices)) return FP_ERR_INVALID_ARG;
  if (ctx16 && !out_proj) return FP_ERR_INVALID_ARG;
  if (base_blocks < 0 || base_blocks > NB) return FP_ERR_INVALID_ARG;
  if (block_stride < 1 || block_offset < 0 || block_offset >= block_stride) return FP_ERR_INVALID_ARG;
  if (!aligned16(x)) return FP_ERR_INVALID_ARG;
  const bool tc = tensor_path(dtype, D);
  if (tc && (!v_t || !w_gu || !aligned16(v_t) || !aligned16(w_gu))) return FP_ERR_INVALID_ARG;
  if (!tc && D > 32 * 256) return FP_ERR_UNSUPPORTED;
  const int cap = std::max(capacity, 1);
  TokenLayout L = token_layout(dtype, M, D, NB, base_blocks, capacity, block_stride, block_offset);
  if (workspace_bytes < L.total)  // a smaller workspace: no decode split
    L = token_layout(dtype, M, D, NB, base_blocks, capacity, block_stride, block_offset, false);
  if (workspace_bytes < L.total) return FP_ERR_WORKSPACE;
  // peer output: the tensor-core path whose contraction stores whole rows (no split-K), checked before any
  // launch so that every rank of a job (same M) falls back together
  if (peer && (!tc || L.nbl == 0 || L.ksplit > 1)) return FP_ERR_UNSUPPORTED;
  int sms;
  FP_TRY(device_info(sms));
  cudaStream_t st = (cudaStream_t)stream;
  int* err = at<int>(workspace, L.err);
  if (cudaMemsetAsync(err, 0, L.zero_bytes, st) != cudaSuccess) return FP_ERR_CUDA;
  const int nbl = L.nbl;
  const bool csr = tc && nbl > 0;
  if (!csr) {
    SimtArgs a{};
    a.x = x; a.k_gate = k_gate; a.k_up = k_up; a.v = v; a.dtype = dtype; a.M = M; a.D = D; a.NB = NB;
    a.base = base_blocks; a.ridx = remote_indices; a.rcnt = remote_counts; a.cap = cap;
    a.active = nbl == 0 ? remote_counts : nullptr; a.n_active = 0;
    a.stride = block_stride; a.offset = block_offset; a.ctx16 = ctx16; a.out_proj = out_proj; a.y = y;
    a.y_f32 = y_f32;
    return launch_simt(a, st);
  }
  stage_mark(0, st);
  RouteArgs r{};
  r.x = x; r.M = M; r.D = D; r.NB = NB; r.temperature = 1.0f;
  r.sel = SelectOut{NB, base_blocks, 1.0f, 0, 0, cap, nullptr, nullptr, nullptr, nullptr};
  r.err = err; r.num_sms = sms;
  r.given_idx = remote_indices; r.given_cnt = remote_counts; r.given_cap = capacity;
  int32_t* key_cnt = at<int32_t>(workspace, L.key_cnt);
  int32_t* pair_tok = at<int32_t>(workspace, L.pair_tok);
  int2* tiles = at<int2>(workspace, L.tiles);
  int32_t* meta = at<int32_t>(workspace, L.meta);
  void* h = at<void>(workspace, L.h);
  r.hzero = static_cast<uint4*>(h); r.hrow_vec = (int64_t)nbl * kBlock * 2 / 16;
  r.key_cnt = key_cnt; r.pair_tok = pair_tok; r.key_cap = L.key_cap;
  r.stride = block_stride; r.offset = block_offset; r.nbl = nbl; r.chunk = L.chunk; r.nkey = L.nkey;
  r.tiles = tiles; r.max_tiles = L.max_tiles; r.meta = meta;
  r.ticket = reinterpret_cast<unsigned int*>(at<char>(workspace, L.err + kTicketOffset));
  FP_TRY(launch_route(r, dtype, st));
  stage_mark(1, st);
  stage_mark(2, st);
  GateUpArgs g{};
  g.x = x; g.w_gu = w_gu; g.M = M; g.D = D; g.Np = NB * kBlock;
  g.tiles = tiles; g.meta = meta; g.key_cnt = key_cnt; g.pair_tok = pair_tok; g.key_cap = L.key_cap;
  g.nbl = nbl; g.stride = block_stride; g.offset = block_offset; g.active = nullptr; g.n_keys = 0;
  g.h = h; g.ldh = (int64_t)nbl * kBlock; g.err = err; g.num_sms = sms;
  if (L.gu_ks > 1) {
    g.gu_ks = L.gu_ks; g.gu_part = at<float>(workspace, L.gu_part); g.max_tiles = L.max_tiles;
  }
  FP_TRY(launch_gateup(g, st));
  stage_mark(3, st);
  DownArgs d{};
  d.h = h; d.v_t = v_t; d.vt_tiled = 1; d.M = M; d.D = D; d.Np = NB * kBlock; d.K = nbl * kBlock; d.bmap = nullptr;
  d.stride = block_stride; d.offset = block_offset; d.ctx16 = ctx16; d.out_proj = out_proj;
  d.out_proj_f32 = dtype == FP_DTYPE_F32; d.y = y; d.y_f32 = y_f32; d.err = err; d.num_sms = sms;
  d.ksplit = L.ksplit; d.y_acc = L.ksplit > 1 ? at<float>(workspace, L.yacc) : nullptr;
  if (M <= 64) {
    d.ktiles = tiles; d.knbl = nbl; d.kcnt = meta;
  }
  if (peer) {
    for (int w = 0; w < peer->world; ++w) d.peer_y[w] = peer->out[w];
    d.peer_rows = peer->rows;
  }
  FP_TRY(launch_down(d, st));
  if (peer) {
    PeerFlags f{};
    for (int w = 0; w < peer->world; ++w) f.flag[w] = peer->flags[w];
    f.world = peer->world;
    FP_TRY(launch_peer_signal(f, peer->epoch, st));
  }
  stage_mark(4, st);
  return FP_OK;
}
}  // namespace

int fp_pattention_routed_fwd(const void* x, int64_t M, int D, int NB, int dtype, const void* k_gate,
                             const void* k_up, const void* v, const void* w_gu, const void* v_t, const void* out_proj,
                             int base_blocks, int capacity, const int32_t* remote_indices,
                             const int32_t* remote_counts, const float* ctx16, int block_stride, int block_offset,
                             void* y, int y_f32, void* workspace, size_t workspace_bytes, void* stream) {
  return routed_fwd_impl(x, M, D, NB, dtype, k_gate, k_up, v, w_gu, v_t, out_proj, base_blocks, capacity,
                         remote_indices, remote_counts, ctx16, block_stride, block_offset, y, y_f32, workspace,
                         workspace_bytes, stream, nullptr);
}

int fp_peer_reduce_supported(int dtype, int64_t M, int D, int NB, int capacity, int block_stride) {
  if (check_common(dtype, M, D, NB) != FP_OK || M <= 0 || block_stride < 1) return 0;
  const TokenLayout L = token_layout(dtype, M, D, NB, 0, std::max(capacity, 0), block_stride, 0);
  return tensor_path(dtype, D) && L.nbl > 0 && L.ksplit <= 1 ? 1 : 0;
}

int fp_pattention_routed_peer_fwd(const void* x, int64_t M, int D, int NB, int dtype, const void* k_gate,
                                  const void* k_up, const void* v, const void* w_gu, const void* v_t,
                                  const void* out_proj, int base_blocks, int capacity, const int32_t* remote_indices,
                                  const int32_t* remote_counts, const float* ctx16, int block_stride,
                                  int block_offset, void* const* peer_out, uint32_t* const* peer_flags, int world,
                                  int64_t rows_per_rank, uint32_t epoch, int y_f32, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  const PeerSpec peer{peer_out, peer_flags, world, rows_per_rank, epoch};
  return routed_fwd_impl(x, M, D, NB, dtype, k_gate, k_up, v, w_gu, v_t, out_proj, base_blocks, capacity,
                         remote_indices, remote_counts, ctx16, block_stride, block_offset, nullptr, y_f32, workspace,
                         workspace_bytes, stream, &peer);
}

int fp_pattention_pooled_fwd(const void* x, int64_t M, int D, int NB, int dtype, const void* k_gate,
                             const void* k_up, const void* v, const void* w_gu, const void* v_t, const int32_t* active,
                             int n_active, const float* ctx16, const void* out_proj, void* y, int y_f32,
                             void* workspace, size_t workspace_bytes, void* stream) {
  FP_TRY(check_common(dtype, M, D, NB));
  if (M == 0) return FP_OK;  // empty batch
  if (!x || !k_gate || !k_up || !v || !active || !y || !workspace || n_active < 0 || n_active > NB)
    return FP_ERR_INVALID_ARG;
  if (ctx16 && !out_proj) return FP_ERR_INVALID_ARG;
  const bool tc = tensor_path(dtype, D);
  if (tc && (!v_t || !w_gu || !aligned16(v_t) || !aligned16(w_gu) || !aligned16(x))) return FP_ERR_INVALID_ARG;
  if (!tc && D > 32 * 256) return FP_ERR_UNSUPPORTED;
  const PooledLayout L = pooled_layout(dtype, M, D, NB, n_active);
  if (workspace_bytes < L.total) return FP_ERR_WORKSPACE;
  int sms;
  FP_TRY(device_info(sms));
  cudaStream_t st = (cudaStream_t)stream;
  int* err = at<int>(workspace, L.err);
  if (cudaMemsetAsync(err, 0, 256, st) != cudaSuccess) return FP_ERR_CUDA;
  if (M == 0) return FP_OK;
  if (!tc || n_active == 0) {
    // CUDA-core path (fp32 or untiled shapes); with no active block only the additive stream remains.
    SimtArgs a{};
    a.x = x; a.k_gate = k_gate; a.k_up = k_up; a.v = v; a.dtype = dtype; a.M = M; a.D = D; a.NB = NB;
    a.active = active; a.n_active = n_active; a.stride = 1; a.offset = 0; a.ctx16 = ctx16;
    a.out_proj = out_proj; a.y = y; a.y_f32 = y_f32;
    return launch_simt(a, st);
  }
  void* h = at<void>(workspace, L.h);
  GateUpArgs g{};
  g.x = x; g.w_gu = w_gu; g.M = M; g.D = D; g.Np = NB * kBlock;
  g.tiles = nullptr; g.meta = nullptr; g.key_cnt = nullptr; g.pair_tok = nullptr; g.key_cap = 0;
  g.nbl = n_active; g.stride = 1; g.offset = 0; g.active = active; g.n_keys = n_active;
  g.h = h; g.ldh = (int64_t)n_active * kBlock; g.err = err; g.num_sms = sms;
  stage_mark(0, st);
  FP_TRY(launch_gateup(g, st));
  stage_mark(1, st);
  DownArgs d{};
  d.h = h; d.v_t = v_t; d.vt_tiled = 1; d.M = M; d.D = D; d.Np = NB * kBlock; d.K = n_active * kBlock; d.bmap = active;
  d.stride = 1; d.offset = 0; d.ctx16 = ctx16; d.out_proj = out_proj; d.out_proj_f32 = dtype == FP_DTYPE_F32;
  d.y = y; d.y_f32 = y_f32; d.err = err; d.num_sms = sms;
  d.ksplit = L.ksplit; d.y_acc = L.ksplit > 1 ? at<float>(workspace, L.yacc) : nullptr;
  FP_TRY(launch_down(d, st));
  stage_mark(2, st);
  return FP_OK;
}

// ---------------------------------------------------------------- function-level Pattention
namespace {
struct SharedLayout {
  size_t err, act, h, yacc, total;
  int ksplit;
  bool tc;
};

// Workspace of fp_pattention_fwd: error word, the all-blocks id list (active = NULL), and for the
// tensor-core path the activations H [M, n_active * 64] and the split-K partials of small batches.
SharedLayout shared_layout(int dtype, int64_t M, int K, int Do, int NB, int n_active) {
  SharedLayout L{};
  Carve c;
  L.err = c.take(256);
  L.act = c.take((size_t)std::max(NB, 1) * 4);
  L.tc = tensor_path(dtype, K) && Do % 64 == 0;
  if (L.tc) {
    L.h = c.take((size_t)M * std::max(n_active, 1) * kBlock * 2);
    L.ksplit = down_ksplit(M, Do, std::max(n_active, 1), layout_sms());
    if (L.ksplit > 1) L.yacc = c.take((size_t)L.ksplit * M * Do * 4);
  }
  L.total = c.off;
  return L;
}
}  // namespace

int fp_pack_pattention_weights(const void* k_gate, const void* k_up, const void* v, int dtype, int Np, int K,
                               int D_out, void* w_gu, void* v_t, void* stream) {
  if (!k_gate || !v || !w_gu || !v_t || Np <= 0 || K <= 0 || D_out <= 0) return FP_ERR_INVALID_ARG;
  if (dtype != FP_DTYPE_BF16) return FP_ERR_UNSUPPORTED;
  if (Np % kBlock || K % 64 || D_out % 64) return FP_ERR_UNSUPPORTED;
  const void* ku = k_up ? k_up : k_gate;  // non-gated forms: the gate rows fill both halves
  if (!aligned16(k_gate) || !aligned16(ku) || !aligned16(w_gu) || !aligned16(v_t)) return FP_ERR_INVALID_ARG;
  int sms;
  FP_TRY(device_info(sms));
  cudaStream_t st = (cudaStream_t)stream;
  FP_TRY(launch_pack_gate_up(k_gate, ku, Np, K, w_gu, st));
  return launch_pack_vt(v, Np, D_out, v_t, st);
}

size_t fp_pattention_workspace_size(int dtype, int64_t M, int K, int Np, int D_out, int n_active) {
  return shared_layout(dtype, std::max<int64_t>(M, 0), K, D_out, std::max(Np / kBlock, 1), std::max(n_active, 0))
      .total;
}

int fp_pattention_fwd(const void* x, int64_t M, int K, int Np, int D_out, int dtype, const void* k_gate,
                      const void* k_up, const void* v, const void* w_gu, const void* v_t, const int32_t* active,
                      int n_active, int activation, void* y, void* workspace, size_t workspace_bytes,
                      void* stream) {
  if (dtype != FP_DTYPE_F32 && dtype != FP_DTYPE_BF16) return FP_ERR_UNSUPPORTED;
  if (M < 0 || K <= 0 || Np <= 0 || D_out <= 0 || Np % kBlock) return FP_ERR_INVALID_ARG;
  if (activation < FP_ACT_SWIGLU || activation > FP_ACT_RELU2) return FP_ERR_INVALID_ARG;
  if (activation == FP_ACT_SWIGLU && !k_up) return FP_ERR_INVALID_ARG;
  if (active && n_active < 0) return FP_ERR_INVALID_ARG;
  if (M > (int64_t)INT32_MAX / 8) return FP_ERR_UNSUPPORTED;
  const int NB = Np / kBlock;
  const int nact = active ? n_active : NB;
  if (M == 0) return FP_OK;
  if (!x || !k_gate || !v || !y || !workspace) return FP_ERR_INVALID_ARG;
  const SharedLayout L = shared_layout(dtype, M, K, D_out, NB, nact);
  if (workspace_bytes < L.total) return FP_ERR_WORKSPACE;
  int sms;
  FP_TRY(device_info(sms));
  cudaStream_t st = (cudaStream_t)stream;
  int* err = at<int>(workspace, L.err);
  if (cudaMemsetAsync(err, 0, 256, st) != cudaSuccess) return FP_ERR_CUDA;
  const int32_t* list = active;
  if (!list) {
    int32_t* all = at<int32_t>(workspace, L.act);
    FP_TRY(launch_iota(all, NB, st));
    list = all;
  }
  const bool tc = L.tc && nact > 0 && w_gu && v_t && aligned16(x) && aligned16(w_gu) && aligned16(v_t) &&
                  aligned16(y);
  if (!tc) {
    // CUDA cores: fp32 (1e-4 tolerance), widths that are not multiples of 64, or no packed layouts
    if (K > 56 * 1024 || D_out > 32 * 256) return FP_ERR_UNSUPPORTED;
    SimtArgs a{};
    a.x = x; a.k_gate = k_gate; a.k_up = k_up; a.v = v; a.dtype = dtype; a.M = M; a.D = K; a.NB = NB;
    a.active = list; a.n_active = nact; a.stride = 1; a.offset = 0; a.ctx16 = nullptr; a.out_proj = nullptr;
    a.y = y; a.y_f32 = 0; a.D_out = D_out; a.act = activation;
    return launch_simt(a, st);
  }
  void* h = at<void>(workspace, L.h);
  GateUpArgs g{};
  g.x = x; g.w_gu = w_gu; g.M = M; g.D = K; g.Np = Np;
  g.tiles = nullptr; g.meta = nullptr; g.key_cnt = nullptr; g.pair_tok = nullptr; g.key_cap = 0;
  g.nbl = nact; g.stride = 1; g.offset = 0; g.active = list; g.n_keys = nact;
  g.h = h; g.ldh = (int64_t)nact * kBlock; g.err = err; g.num_sms = sms; g.act = activation;
  FP_TRY(launch_gateup(g, st));
  DownArgs d{};
  d.h = h; d.v_t = v_t; d.vt_tiled = 1; d.M = M; d.D = D_out; d.Np = Np; d.K = nact * kBlock; d.bmap = list;
  d.stride = 1; d.offset = 0; d.ctx16 = nullptr; d.out_proj = nullptr; d.out_proj_f32 = 0;
  d.y = y; d.y_f32 = 0; d.err = err; d.num_sms = sms;
  d.ksplit = L.ksplit; d.y_acc = L.ksplit > 1 ? at<float>(workspace, L.yacc) : nullptr;
  return launch_down(d, st);
}

size_t fp_block_energy_workspace_size(int64_t M, int NB) {
  Carve c;
  c.take(256);                                   // error word
  c.take((size_t)std::max(NB, 1) * 4);           // active ids 0..NB-1
  c.take((size_t)4 * std::max<int64_t>(M, 0) * std::max(NB, 1) * 4);  // per-quarter partial energies
  return c.off;
}

int fp_block_energy(const void* x, int64_t M, int D, int NB, int dtype, const void* w_gu, const float* vnorm,
                    float* energy, void* workspace, size_t workspace_bytes, void* stream) {
  FP_TRY(check_common(dtype, M, D, NB));
  if (M == 0) return FP_OK;
  if (!x || !w_gu || !vnorm || !energy || !workspace) return FP_ERR_INVALID_ARG;
  if (!tensor_path(dtype, D)) return FP_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(w_gu)) return FP_ERR_INVALID_ARG;
  if (workspace_bytes < fp_block_energy_workspace_size(M, NB)) return FP_ERR_WORKSPACE;
  int sms;
  FP_TRY(device_info(sms));
  cudaStream_t st = (cudaStream_t)stream;
  Carve c;
  int* err = at<int>(workspace, c.take(256));
  int32_t* act = at<int32_t>(workspace, c.take((size_t)NB * 4));
  float* part = at<float>(workspace, c.take((size_t)4 * M * NB * 4));
  if (cudaMemsetAsync(err, 0, 256, st) != cudaSuccess) return FP_ERR_CUDA;
  FP_TRY(launch_iota(act, NB, st));
  GateUpArgs g{};
  g.x = x; g.w_gu = w_gu; g.M = M; g.D = D; g.Np = NB * kBlock;
  g.tiles = nullptr; g.meta = nullptr; g.key_cnt = nullptr; g.pair_tok = nullptr; g.key_cap = 0;
  g.nbl = NB; g.stride = 1; g.offset = 0; g.active = act; g.n_keys = NB;
  g.h = nullptr; g.ldh = 0; g.energy = part; g.err = err; g.num_sms = sms;
  FP_TRY(launch_gateup(g, st));
  return launch_energy_combine(part, M, NB, vnorm, energy, st);
}

int fp_set_stage_events(void* const* events, int n_events) {
  if (n_events < 0 || n_events > 8 || (n_events > 0 && !events)) return FP_ERR_INVALID_ARG;
  for (int i = 0; i < 8; ++i) g_stage_events[i] = i < n_events ? (cudaEvent_t)events[i] : nullptr;
  g_n_stage = n_events;
  return FP_OK;
}

// ---------------------------------------------------------------- union-contraction layers
int fp_param_blocks_16d(const void* P, const void* k_proj, const void* v_proj, int dtype, int64_t N, int D,
                        float* k_blocks, float* v_blocks, void* stream) {
  if (dtype != FP_DTYPE_F32 && dtype != FP_DTYPE_BF16) return FP_ERR_UNSUPPORTED;
  if (!P || !k_proj || !v_proj || !k_blocks || !v_blocks || N <= 0 || D <= 0 || N % 64 != 0) return FP_ERR_INVALID_ARG;
  if (N / 64 > INT32_MAX) return FP_ERR_UNSUPPORTED;
  int sms;
  FP_TRY(device_info(sms));
  return launch_param_blocks_16d(P, k_proj, v_proj, dtype, N, D, k_blocks, v_blocks, (cudaStream_t)stream);
}

int fp_cosine_block_scores(const void* x, const void* q_proj, const float* k_blocks, int dtype, int64_t M, int D,
                           int NB, float* scores, float* q16, void* stream) {
  FP_TRY(check_common(dtype, M, D, NB));
  if (!x || !q_proj || !k_blocks || !scores) return FP_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(q_proj)) return FP_ERR_INVALID_ARG;
  int sms;
  FP_TRY(device_info(sms));
  return launch_router_scores(x, q_proj, k_blocks, dtype, M, D, NB, 1.0f, scores, q16, (cudaStream_t)stream,
                              k_blocks);
}

int fp_select_remote_top_p(const float* scores, int64_t M, int NB, int base, float top_p, int max_remote,
                           int capacity, int32_t* remote_indices, int32_t* remote_counts, float* stats,
                           void* stream) {
  if (M < 0 || NB <= 0 || base < 0 || base > NB || capacity < 0 || max_remote < 0) return FP_ERR_INVALID_ARG;
  if (!scores || !remote_counts || (capacity > 0 && !remote_indices)) return FP_ERR_INVALID_ARG;
  if (NB - base > 1024) return FP_ERR_UNSUPPORTED;
  int sms;
  FP_TRY(device_info(sms));
  cudaStream_t st = (cudaStream_t)stream;
  if (M == 0) return FP_OK;
  if (NB == base) {  // no remote columns: the reference keeps the base blocks only (block_matmul.py:202-205)
    if (cudaMemsetAsync(remote_counts, 0, (size_t)M * 4, st) != cudaSuccess) return FP_ERR_CUDA;
    if (capacity > 0 && cudaMemsetAsync(remote_indices, 0, (size_t)M * capacity * 4, st) != cudaSuccess)
      return FP_ERR_CUDA;
    return FP_OK;
  }
  SelectOut o{NB - base, 0, top_p, 0, max_remote, capacity, remote_indices, remote_counts, nullptr, stats};
  o.ld = NB;
  o.id_offset = base;
  o.fast = 1;
  return launch_select_out(scores + base, M, 1.0f, o, nullptr, st);
}

int fp_union_blocks(const int32_t* remote_indices, const int32_t* remote_counts, int64_t M, int capacity, int NB,
                    int base, int32_t* blocks, int32_t* n_active, void* stream) {
  if (M < 0 || capacity < 0 || NB <= 0 || base < 0 || !blocks || !n_active) return FP_ERR_INVALID_ARG;
  if (M > 0 && capacity > 0 && (!remote_indices || !remote_counts)) return FP_ERR_INVALID_ARG;
  int sms;
  FP_TRY(device_info(sms));
  return launch_union(remote_indices, remote_counts, M, capacity, NB, std::min(base, NB), blocks, n_active,
                      (cudaStream_t)stream);
}

namespace {
// Split-K factor of the BlockSparseLinear contraction on the one-SM tensor-core kernel (batches under 256
// tokens): the output tiles of at most max_active blocks cannot occupy the GPU, so the contraction over
// D_in is split (as down_ksplit does for the MLP's down projection).
int bsl_ksplit(int dtype, int64_t M, int D_in, int out_features, int max_active, int sms) {
  if (!tensor_path(dtype, D_in) || M >= 2 * kTileM) return 1;
  const int NB = out_features / kBlock;
  const int nact = max_active > 0 ? std::min(max_active, NB) : NB;
  return down_ksplit(M, nact * kBlock, D_in / kTileK, sms);
}
size_t bsl_workspace(int ks, int64_t M, int out_features) {
  return ks > 1 ? align_up(FP_VARIANT_WORKSPACE_MIN) + (size_t)ks * M * out_features * 4
                : (size_t)FP_VARIANT_WORKSPACE_MIN;
}
}  // namespace

size_t fp_block_sparse_linear_workspace_size(int dtype, int64_t M, int D_in, int out_features, int max_active) {
  if (M <= 0 || D_in <= 0 || out_features <= 0) return FP_VARIANT_WORKSPACE_MIN;
  return bsl_workspace(bsl_ksplit(dtype, M, D_in, out_features, max_active, layout_sms()), M, out_features);
}

int fp_pack_blocked_weight(const void* weight, int rows, int cols, void* out, void* stream) {
  if (!weight || !out || rows <= 0 || cols <= 0 || rows % 64 || cols % 64) return FP_ERR_INVALID_ARG;
  if (!aligned16(weight) || !aligned16(out)) return FP_ERR_INVALID_ARG;
  return launch_pack_blocked(weight, rows, cols, out, (cudaStream_t)stream);
}

namespace {
int bsl_fwd(const void* x, int64_t M, int D_in, const void* weight, const void* weight_blocked, const void* bias,
            int out_features, int dtype, const int32_t* blocks, const int32_t* n_active, int max_active,
            const float* ctx16, const void* out_proj, void* out, void* workspace, size_t workspace_bytes,
            void* stream) {
  if (dtype != FP_DTYPE_F32 && dtype != FP_DTYPE_BF16) return FP_ERR_UNSUPPORTED;
  if (M < 0 || D_in <= 0 || out_features <= 0 || out_features % 64 != 0) return FP_ERR_INVALID_ARG;
  if (!x || !weight || !blocks || !n_active || !out || (ctx16 && !out_proj)) return FP_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < FP_VARIANT_WORKSPACE_MIN) return FP_ERR_WORKSPACE;
  if (M > (int64_t)INT32_MAX / 8) return FP_ERR_UNSUPPORTED;
  int sms;
  FP_TRY(device_info(sms));
  cudaStream_t st = (cudaStream_t)stream;
  if (M == 0) return FP_OK;
  const int NB = out_features / 64;
  int* err = static_cast<int*>(workspace);
  if (cudaMemsetAsync(workspace, 0, FP_VARIANT_WORKSPACE_MIN, st) != cudaSuccess) return FP_ERR_CUDA;
  const int f32 = dtype == FP_DTYPE_F32;
  if (tensor_path(dtype, D_in) && aligned16(x) && aligned16(weight) && aligned16(out) &&
      (!out_proj || aligned16(out_proj))) {
    const int ks = bsl_ksplit(dtype, M, D_in, out_features, max_active, sms);
    if (workspace_bytes < bsl_workspace(ks, M, out_features)) return FP_ERR_WORKSPACE;
    DownArgs d{};
    d.h = x; d.v_t = weight; d.M = M; d.D = out_features; d.Np = D_in; d.K = D_in;
    d.stride = 1; d.offset = 0;
    d.ctx16 = ctx16; d.out_proj = out_proj; d.out_proj_f32 = 0;
    d.y = out; d.y_f32 = 0; d.ksplit = ks; d.err = err; d.num_sms = sms;
    d.y_acc = ks > 1 ? reinterpret_cast<float*>(static_cast<char*>(workspace) + align_up(FP_VARIANT_WORKSPACE_MIN))
                     : nullptr;
    d.nmap = blocks; d.omap = blocks; d.ncnt = n_active; d.bias = bias; d.bias_f32 = 0; d.ldy = out_features;
    if (weight_blocked && aligned16(weight_blocked)) {
      d.v_t = weight_blocked;
      d.vt_blocked = 1;
    }
    FP_TRY(launch_down(d, st));
  } else {
    MappedGemm g{};
    g.a = x; g.lda = D_in; g.a_f32 = f32;
    g.b = weight; g.ldb = D_in; g.b_f32 = f32; g.nn = 0;
    g.M = M; g.K = D_in; g.N = out_features;
    g.nmap = blocks; g.omap = blocks; g.ncnt = n_active;
    g.bias = bias; g.bias_f32 = f32;
    g.ctx16 = ctx16; g.out_proj = out_proj; g.out_proj_f32 = f32;
    g.y = out; g.ldy = out_features; g.y_f32 = f32;
    FP_TRY(launch_mapped_gemm_simt(g, st));
  }
  return launch_fill_inactive(blocks, n_active, NB, M, ctx16, out_proj, dtype, out, out_features, sms, st);
}
}  // namespace

int fp_block_sparse_linear_fwd(const void* x, int64_t M, int D_in, const void* weight, const void* bias,
                               int out_features, int dtype, const int32_t* blocks, const int32_t* n_active,
                               int max_active, const float* ctx16, const void* out_proj, void* out, void* workspace,
                               size_t workspace_bytes, void* stream) {
  return bsl_fwd(x, M, D_in, weight, nullptr, bias, out_features, dtype, blocks, n_active, max_active, ctx16,
                 out_proj, out, workspace, workspace_bytes, stream);
}

int fp_block_sparse_linear_blocked_fwd(const void* x, int64_t M, int D_in, const void* weight,
                                       const void* weight_blocked, const void* bias, int out_features, int dtype,
                                       const int32_t* blocks, const int32_t* n_active, int max_active,
                                       const float* ctx16, const void* out_proj, void* out, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  if (weight_blocked && (dtype != FP_DTYPE_BF16 || D_in % 64)) return FP_ERR_INVALID_ARG;
  return bsl_fwd(x, M, D_in, weight, weight_blocked, bias, out_features, dtype, blocks, n_active, max_active, ctx16,
                 out_proj, out, workspace, workspace_bytes, stream);
}

namespace {
struct TfLayout {
  size_t s, p, total;
};
TfLayout tf_layout(int dtype, int64_t M, int Np) {
  TfLayout L{};
  Carve c;
  c.take(FP_VARIANT_WORKSPACE_MIN);  // device error word
  // scores and activation weights: bf16 on the tensor-core path, fp32 on the CUDA-core path (which bf16
  // layers also take for shapes the tensor path does not tile), so 4 bytes per element cover both
  (void)dtype;
  L.s = c.take((size_t)M * Np * 4);
  L.p = c.take((size_t)M * Np * 4);
  L.total = c.off;
  return L;
}
}  // namespace

size_t fp_tokenformer_workspace_size(int dtype, int64_t M, int num_param_tokens) {
  return tf_layout(dtype, std::max<int64_t>(M, 0), std::max(num_param_tokens, 0)).total;
}

int fp_tokenformer_fwd(const void* x, int64_t M, int D_in, const void* k_param, const void* v_param,
                       const void* v_param_t, int num_param_tokens, int D_out, int dtype, int activation,
                       const int32_t* blocks, const int32_t* n_active, const float* ctx16, const void* out_proj,
                       void* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != FP_DTYPE_F32 && dtype != FP_DTYPE_BF16) return FP_ERR_UNSUPPORTED;
  const int Np = num_param_tokens;
  if (M < 0 || D_in <= 0 || D_out <= 0 || Np <= 0 || Np % 64 != 0) return FP_ERR_INVALID_ARG;
  if (activation != 0 && activation != 1) return FP_ERR_INVALID_ARG;
  if (!x || !k_param || !v_param || !blocks || !n_active || !out || (ctx16 && !out_proj)) return FP_ERR_INVALID_ARG;
  if (M > (int64_t)INT32_MAX / 8) return FP_ERR_UNSUPPORTED;
  const TfLayout L = tf_layout(dtype, M, Np);
  if (!workspace || workspace_bytes < L.total) return FP_ERR_WORKSPACE;
  int sms;
  FP_TRY(device_info(sms));
  cudaStream_t st = (cudaStream_t)stream;
  if (M == 0) return FP_OK;
  char* ws = static_cast<char*>(workspace);
  int* err = reinterpret_cast<int*>(ws);
  void* S = ws + L.s;
  void* P = ws + L.p;
  if (cudaMemsetAsync(workspace, 0, FP_VARIANT_WORKSPACE_MIN, st) != cudaSuccess) return FP_ERR_CUDA;
  const int f32 = dtype == FP_DTYPE_F32;
  const float div = sqrtf((float)D_in);  // math.sqrt(in_features) as the fp32 divisor (tokenformer.py:104)
  const bool tc = tensor_path(dtype, D_in) && D_out % 64 == 0 && v_param_t && aligned16(x) && aligned16(k_param) &&
                  aligned16(v_param_t) && aligned16(out) && (!out_proj || aligned16(out_proj));
  if (tc) {
    DownArgs g1{};  // S[:, j*64 + c] = x . k_param[blocks[j]*64 + c]
    g1.h = x; g1.v_t = k_param; g1.M = M; g1.D = Np; g1.Np = D_in; g1.K = D_in; g1.stride = 1;
    g1.y = S; g1.y_f32 = 0; g1.ksplit = 1; g1.err = err; g1.num_sms = sms;  // bf16 scores
    g1.nmap = blocks; g1.ncnt = n_active; g1.ldy = Np;
    FP_TRY(launch_down(g1, st));
    FP_TRY(launch_rowact(S, 1, Np, M, n_active, activation, div, P, Np, 0, st, Np));
    DownArgs g2{};  // out = P[:, :64 n] . v_param[blocks] + ctx16 . out_proj^T
    g2.h = P; g2.v_t = v_param_t; g2.M = M; g2.D = D_out; g2.Np = Np; g2.K = Np; g2.stride = 1;
    g2.bmap = blocks; g2.kcnt = n_active;
    g2.ctx16 = ctx16; g2.out_proj = out_proj; g2.out_proj_f32 = 0;
    g2.y = out; g2.y_f32 = 0; g2.ksplit = 1; g2.err = err; g2.num_sms = sms; g2.ldy = D_out;
    return launch_down(g2, st);
  }
  MappedGemm g1{};
  g1.a = x; g1.lda = D_in; g1.a_f32 = f32;
  g1.b = k_param; g1.ldb = D_in; g1.b_f32 = f32; g1.nn = 0;
  g1.M = M; g1.K = D_in; g1.N = Np;
  g1.nmap = blocks; g1.ncnt = n_active;
  g1.y = S; g1.ldy = Np; g1.y_f32 = 1;
  FP_TRY(launch_mapped_gemm_simt(g1, st));
  FP_TRY(launch_rowact(S, 0, Np, M, n_active, activation, div, P, Np, 1, st, Np));
  MappedGemm g2{};
  g2.a = P; g2.lda = Np; g2.a_f32 = 1;
  g2.b = v_param; g2.ldb = D_out; g2.b_f32 = f32; g2.nn = 1;
  g2.M = M; g2.K = Np; g2.N = D_out;
  g2.kmap = blocks; g2.kcnt = n_active;
  g2.ctx16 = ctx16; g2.out_proj = out_proj; g2.out_proj_f32 = f32;
  g2.y = out; g2.ldy = D_out; g2.y_f32 = f32;
  return launch_mapped_gemm_simt(g2, st);
}

int fp_transpose(const void* src, int64_t rows, int64_t cols, int dtype, void* dst, void* stream) {
  if (dtype != FP_DTYPE_F32 && dtype != FP_DTYPE_BF16) return FP_ERR_UNSUPPORTED;
  if (!src || !dst || rows < 0 || cols < 0) return FP_ERR_INVALID_ARG;
  int sms;
  FP_TRY(device_info(sms));
  return launch_transpose(src, rows, cols, dtype, dst, (cudaStream_t)stream);
}

int fp_device_error(void* workspace, void* stream, int* code) {
  if (!workspace) return FP_ERR_INVALID_ARG;
  int host = 0;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemcpyAsync(&host, workspace, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return FP_ERR_CUDA;
  if (code) *code = host;
  if (host != 0 && cudaMemsetAsync(workspace, 0, sizeof(int), st) != cudaSuccess) return FP_ERR_CUDA;
  return host == 0 ? FP_OK : FP_ERR_TIMEOUT;
}

}  // extern "C"
