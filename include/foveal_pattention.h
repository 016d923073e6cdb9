/*
 * foveal_pattention.h — C ABI of libfovealpatt.so, the B200 (sm_100a) implementation of the Foveal
 * Pattention MLP forward: 16-D router, top-p block selection and the gated block-sparse SwiGLU
 * contraction with the 16-D additive stream.
 *
 * The reference (kreasof-ai/foveal-sparse-indexer) has no native interface: its hot path is the
 * Python module FovealPattentionMLP and the functions it calls.  Each entry point below names the
 * reference function it replaces (paths relative to that project).
 *
 * Conventions (all entry points):
 *   - All tensor pointers are DEVICE pointers, row-major and contiguous, 16-byte aligned.
 *   - dtype: FP_DTYPE_F32 or FP_DTYPE_BF16 for x and all weights of one call.
 *   - The caller allocates every output and the workspace (size from the *_workspace_size queries).
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Work is only enqueued: no entry
 *     point synchronizes the host except fp_device_error.
 *   - Return value: FP_OK (0) or an fp_status code.  No exception crosses the ABI.
 *   - Thread-safe as long as concurrent calls use different workspaces.
 *   - Kernels never wait unboundedly: a wait that runs out records a code that fp_device_error
 *     returns as FP_ERR_TIMEOUT.
 */
#ifndef FOVEAL_PATTENTION_H_
#define FOVEAL_PATTENTION_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FP_ABI_VERSION 1

#if defined(__GNUC__)
#define FP_API __attribute__((visibility("default")))
#else
#define FP_API
#endif

typedef enum fp_status {
  FP_OK = 0,
  FP_ERR_INVALID_ARG = 1,  /* null pointer, bad shape or parameter, misaligned pointer */
  FP_ERR_UNSUPPORTED = 2,  /* dtype / shape combination not implemented */
  FP_ERR_WORKSPACE = 3,    /* workspace too small */
  FP_ERR_CUDA = 4,         /* a CUDA runtime call or kernel launch failed */
  FP_ERR_DEVICE = 5,       /* current device is not an sm_100 GPU */
  FP_ERR_TIMEOUT = 6       /* a kernel's bounded wait ran out (reported by fp_device_error) */
} fp_status;

typedef enum fp_dtype { FP_DTYPE_F32 = 0, FP_DTYPE_BF16 = 1 } fp_dtype;

/* Activations of fp_pattention_fwd, numbered like the reference's ACTIVATION_CODE
 * (pattention_triton.py:121, :172-191): SwiGLU silu(g) * u, SiLU silu(g), GELU (erf form, as
 * F.gelu in _pytorch_pattention_fallback, :303), ReLU, squared ReLU. */
typedef enum fp_activation {
  FP_ACT_SWIGLU = 0,
  FP_ACT_SILU = 1,
  FP_ACT_GELU = 2,
  FP_ACT_RELU = 3,
  FP_ACT_RELU2 = 4
} fp_activation;

/* ABI version (FP_ABI_VERSION of the built library). */
FP_API int fp_abi_version(void);

/* Static description of a status code. */
FP_API const char* fp_status_string(int status);

/*
 * Router scores.  Replaces FovealPattentionMLP.compute_router_scores
 * (foveal_indexer/foveal_pattention.py:257-262):
 *   scores[m, b] = (rms_norm(x[m] . q_proj^T) . block_keys[b]) / sqrt(16)        (fp32 out)
 * x [M, D], q_proj [16, D], block_keys [NB, 16] in `dtype`; q16 (optional) [M, 16] fp32 receives the
 * normalised 16-D queries (FovealIndexer.compute_query_16d, foveal_indexer/core.py:214-223).
 * D must be a multiple of 8; NB <= 1024.
 */
FP_API int fp_router_scores(const void* x, const void* q_proj, const void* block_keys, int dtype, int64_t M,
                     int D, int NB, float* scores, float* q16, void* stream);

/*
 * Adaptive top-p block selection, non-causal, with `base_blocks` always-on leading blocks.  Replaces
 * select_blocks(block_scores, causal=False, local_window_blocks=base_blocks, top_p, min_remote_blocks,
 * max_remote_blocks, remote_capacity) (foveal_indexer/core.py:46-160, branch :90-99) and, when ctx16
 * is given, the additive-stream context softmax(S / T) . K_16 (foveal_pattention.py:339-340).
 *   scores         [M, NB] fp32 pre-softmax scores S (divided by `temperature` before the softmax)
 *   remote_indices [M, capacity] int32: block ids by descending probability, ties to the lower id
 *   remote_counts  [M] int32: number of selected remote blocks
 *   block_keys_f32 [NB, 16] fp32 and ctx16 [M, 16] fp32: both NULL or both set
 *   stats          optional float[3] accumulated in place: sum of (count >= K_max), sum of counts,
 *                  sum of (count == 0); divide by M for cap_rate, mean_remote_blocks, base_only_rate
 */
FP_API int fp_select_blocks(const float* scores, int64_t M, int NB, int base_blocks, float top_p, int min_remote,
                     int max_remote, int capacity, float temperature, int32_t* remote_indices,
                     int32_t* remote_counts, const float* block_keys_f32, float* ctx16, float* stats,
                     void* stream);

/*
 * Pooled routing: one active set for the whole call (foveal_pattention.py:292-303 training,
 * :310-321 eval).  active[0..base) = 0..base-1, then `remote_blocks` ids by descending pooled score.
 *   mode 0 (eval):  pooled query rms_norm(q_proj . mean_t(x)), scores = q . K_16^T (no 1/sqrt(16))
 *   mode 1 (train): token-mean of `token_scores` [M, NB] (fp32, from fp_router_scores)
 * mean_scores (optional) [NB] fp32 receives the pooled scores.  Workspace: fp_pooled_workspace_size.
 */
FP_API int fp_pooled_route(const void* x, const void* q_proj, const void* block_keys, int dtype, int64_t M, int D,
                    int NB, int base_blocks, int remote_blocks, int mode, const float* token_scores,
                    int32_t* active, float* mean_scores, void* workspace, size_t workspace_bytes,
                    void* stream);

/*
 * Weight layouts for the tensor-core path (bf16), derived from the reference parameters
 * (FovealPattentionMLP.k_gate / k_up / v, foveal_pattention.py:86-88; v stores W_down^T, :169).  Both
 * are tile-contiguous, so that each pipeline stage of the contraction kernels streams one contiguous
 * tile:
 *   w_gu (2 * Np * D elements): per parameter block b, 128 packed rows (rows 32q..32q+15 = k_gate
 *        channels 16q..16q+15 and rows 32q+16..32q+31 = k_up channels 16q..16q+15 of the block, q = 0..3);
 *        the 128 x 64 tile of columns [kb*64, +64) is contiguous at element offset (kb * Np/64 + b) * 8192
 *        (k-block-major: a block's tiles are spread over the whole buffer)
 *   v_t  (ceil(D / 256) * 256 * Np elements): v transposed in 256 x 64 tiles; the tile of output columns
 *        [n*256, +256) and parameter tokens [b*64, +64) is contiguous (row = output column, 64 elements)
 *        at element offset (n * Np/64 + b) * 16384; columns past D are zero
 * Call once per weight update.  Np % 64 == 0, D % 64 == 0.
 */
FP_API int fp_pack_weights(const void* k_gate, const void* k_up, const void* v, int dtype, int Np, int D,
                           void* w_gu, void* v_t, void* stream);

/* Workspace bytes of fp_pattention_token_fwd (block_stride = 1 unless blocks are sharded). */
FP_API size_t fp_token_workspace_size(int dtype, int64_t M, int D, int NB, int base_blocks, int max_remote,
                               int block_stride);

/* Workspace bytes of fp_pattention_pooled_fwd and fp_pooled_route. */
FP_API size_t fp_pooled_workspace_size(int dtype, int64_t M, int D, int NB, int n_active);

/*
 * Per-token routed forward (router + selection + gated contraction + additive stream), the
 * composition compute_router_scores -> select_blocks(non-causal, base) -> per-token Pattention over
 * base ∪ selected (pattention_triton.py:280-311, "swiglu", block_n = 64) -> + out_proj_16d(softmax(S/T) K_16)
 * (foveal_pattention.py:257-262, core.py:46-160, foveal_pattention.py:338-342).
 *   x [M, D]; k_gate, k_up, v [Np, D] (Np = NB * 64); w_gu and v_t (tile-contiguous) from
 *   fp_pack_weights (bf16 tensor-core path; may be NULL for fp32); q_proj [16, D]; block_keys [NB, 16];
 *   out_proj [D, 16]; all in `dtype`.
 *   additive: 1 adds the additive stream.
 *   block_stride / block_offset: this call computes only blocks b with b % block_stride == block_offset
 *   (parameter-block sharding across GPUs; 1 / 0 = all blocks).  Routing still covers all blocks.
 *   y [M, D]: `dtype`, or fp32 when y_f32 = 1 (partial sums of a block shard).
 *   remote_indices [M, max_remote] int32, remote_counts [M] int32, scores [M, NB] fp32: optional
 *   outputs (NULL = keep inside the workspace).
 */
FP_API int fp_pattention_token_fwd(const void* x, int64_t M, int D, int NB, int dtype, const void* k_gate,
                            const void* k_up, const void* v, const void* w_gu, const void* v_t, const void* q_proj,
                            const void* block_keys, const void* out_proj, int base_blocks, float top_p,
                            int min_remote, int max_remote, float temperature, int additive,
                            int block_stride, int block_offset, void* y, int y_f32,
                            int32_t* remote_indices, int32_t* remote_counts, float* scores,
                            void* workspace, size_t workspace_bytes, void* stream);

/*
 * The token-routed forward split in two, for parameter-block sharding with the routing itself split
 * over the ranks: each rank routes only its slice of the tokens (fp_route_tokens: the projection, scores
 * and select_blocks of fp_pattention_token_fwd), the ranks exchange the routes (an all-gather), and each
 * rank runs the contraction of its blocks for all tokens from the given routes (fp_pattention_routed_fwd:
 * block lists, gate/up, down and the additive stream of the rows whose ctx16 is given).  Together they
 * replace the same reference functions as fp_pattention_token_fwd.
 *   fp_route_tokens: remote_indices [M, max_remote] int32, remote_counts [M] int32, ctx16 [M, 16] fp32
 *   (softmax(S/T) . K_16, may be NULL), scores [M, NB] fp32 (may be NULL); workspace of
 *   fp_route_workspace_size(M) bytes.
 *   fp_pattention_routed_fwd: remote_indices [M, capacity], remote_counts [M] as written by
 *   fp_route_tokens (ids outside [0, NB) are reported in the device error word and skipped); ctx16 [M, 16]
 *   or NULL (rows of zeros add nothing); block_stride / block_offset and y / y_f32 as in
 *   fp_pattention_token_fwd; workspace of fp_token_workspace_size(dtype, M, D, NB, base_blocks, capacity,
 *   block_stride) bytes.
 */
FP_API size_t fp_route_workspace_size(int64_t M);
FP_API int fp_route_tokens(const void* x, int64_t M, int D, int NB, int dtype, const void* q_proj,
                           const void* block_keys, int base_blocks, float top_p, int min_remote, int max_remote,
                           float temperature, int32_t* remote_indices, int32_t* remote_counts, float* ctx16,
                           float* scores, void* workspace, size_t workspace_bytes, void* stream);
FP_API int fp_pattention_routed_fwd(const void* x, int64_t M, int D, int NB, int dtype, const void* k_gate,
                                    const void* k_up, const void* v, const void* w_gu, const void* v_t,
                                    const void* out_proj, int base_blocks, int capacity,
                                    const int32_t* remote_indices, const int32_t* remote_counts, const float* ctx16,
                                    int block_stride, int block_offset, void* y, int y_f32, void* workspace,
                                    size_t workspace_bytes, void* stream);

/*
 * Peer-memory reduce-scatter of the parameter-block-sharded forward (one process per GPU; GPUs with
 * peer access over NVLink / NVSwitch).  Replaces the NCCL reduce-scatter after the contraction: each rank's
 * down projection stores the partial rows of token slice o directly into rank o's receive buffer while
 * it computes, then raises its flag there; each rank's fp_peer_combine waits for every rank's flag and
 * sums its slots in rank order.
 *   fp_peer_alloc: a zeroed device buffer of `bytes` and its IPC handle (FP_PEER_HANDLE_BYTES written to
 *   handle); fp_peer_open maps another process's buffer from its handle (fp_peer_close unmaps it);
 *   fp_peer_free releases a buffer of fp_peer_alloc.
 *   Receive buffer layout (bytes): [0, FP_PEER_FLAG_BYTES) flags uint32[world] (flag w = the last epoch
 *   whose partial rank w finished storing here), then two parities x world slots x rows x D partials
 *   (bf16, or fp32 with y_f32).  Call e writes parity e % 2; epochs increase by one per call.
 *   fp_pattention_routed_peer_fwd: fp_pattention_routed_fwd (same inputs, M = world * rows_per_rank)
 *   whose output rows go to peer_out[o] (this rank's slot of parity e % 2 on rank o; row r of the batch
 *   to row r - o * rows_per_rank of rank o = r / rows_per_rank), followed by peer_flags[o] = epoch
 *   (this rank's flag word on rank o, release at system scope).  Returns FP_ERR_UNSUPPORTED before any
 *   launch when the shape takes the CUDA-core path or a split contraction (small batches): callers fall
 *   back to the collective.
 *   fp_peer_combine: y [rows, D] (bf16, or fp32 with y_f32) = sum over w in rank order of recv's slot w
 *   (recv = this rank's buffer at the parity of `epoch`), after every flags[w] >= epoch; a wait longer
 *   than the kernels' wait limit (2 s) is reported as FP_ERR_TIMEOUT by fp_device_error(workspace) and leaves y
 *   unwritten.  workspace: at least 256 bytes (error word).
 */
#define FP_PEER_HANDLE_BYTES 64
#define FP_PEER_FLAG_BYTES 256u
FP_API int fp_peer_alloc(size_t bytes, void** ptr, void* handle);
FP_API int fp_peer_open(const void* handle, void** ptr);
FP_API int fp_peer_close(void* ptr);
FP_API int fp_peer_free(void* ptr);
/* 1 when fp_pattention_routed_peer_fwd takes this shape (the tensor-core path with an unsplit
 * contraction), else 0: callers pick the peer path or the collective before exchanging anything. */
FP_API int fp_peer_reduce_supported(int dtype, int64_t M, int D, int NB, int capacity, int block_stride);
FP_API int fp_pattention_routed_peer_fwd(const void* x, int64_t M, int D, int NB, int dtype, const void* k_gate,
                                         const void* k_up, const void* v, const void* w_gu, const void* v_t,
                                         const void* out_proj, int base_blocks, int capacity,
                                         const int32_t* remote_indices, const int32_t* remote_counts,
                                         const float* ctx16, int block_stride, int block_offset,
                                         void* const* peer_out, uint32_t* const* peer_flags, int world,
                                         int64_t rows_per_rank, uint32_t epoch, int y_f32, void* workspace,
                                         size_t workspace_bytes, void* stream);
FP_API int fp_peer_combine(const void* recv, const uint32_t* flags, int world, int64_t rows, int D, int in_f32,
                           uint32_t epoch, void* y, int y_f32, void* workspace, size_t workspace_bytes,
                           void* stream);
/*
 * Small tables every rank holds (the routes of the split routing): fp_peer_put writes the same `bytes`
 * (a multiple of 16, 16-byte aligned) from src to dst[w] on every rank w; fp_peer_signal then raises this
 * rank's flag on every rank (flags[w] = this rank's flag word on rank w, release at system scope, after
 * every store of the stream so far); fp_peer_wait (bounded, like fp_peer_combine's wait; its error word in
 * `workspace`) orders the stream's later work after every flags[w] >= epoch.  The route exchange of the
 * block-sharded forward uses them in place of an all-gather.
 */
FP_API int fp_peer_put(const void* src, size_t bytes, void* const* dst, int world, void* stream);
FP_API int fp_peer_signal(uint32_t* const* flags, int world, uint32_t epoch, void* stream);
FP_API int fp_peer_wait(const uint32_t* flags, int world, uint32_t epoch, void* workspace, size_t workspace_bytes,
                        void* stream);

/*
 * Pooled forward over one shared active set.  Replaces the active-block execution of
 * FovealPattentionMLP.forward (foveal_pattention.py:115-122 gather, :329-335 SwiGLU) and the
 * training-mode additive stream (:338-342) when ctx16 is given.
 *   active [n_active] int32 device ids; ctx16 [M, 16] fp32 (softmax(S/T) K_16, from fp_select_blocks
 *   with capacity 0) or NULL; other tensors as in fp_pattention_token_fwd.
 */
FP_API int fp_pattention_pooled_fwd(const void* x, int64_t M, int D, int NB, int dtype, const void* k_gate,
                             const void* k_up, const void* v, const void* w_gu, const void* v_t, const int32_t* active,
                             int n_active, const float* ctx16, const void* out_proj, void* y, int y_f32,
                             void* workspace, size_t workspace_bytes, void* stream);

/*
 * Function-level Pattention with one active-block list shared by every token: replaces
 * triton_pattention(x, k_gate, v, k_up=None, active_blocks=None, activation, block_n=64)
 * (pattention_triton.py:204-277; semantics of _pytorch_pattention_fallback, :280-311).
 *   y = act(x . K_gate[A]^T, x . K_up[A]^T) . V[A],  A = the rows of blocks active[0 .. n_active)
 *   x [M, K]; k_gate, k_up [Np, K]; v [Np, D_out]; y [M, D_out]; all in `dtype`.
 *   k_up may be NULL unless activation == FP_ACT_SWIGLU (the other activations read k_gate only).
 *   active [n_active] int32 device ids, or NULL for every block (n_active ignored).
 *   w_gu, v_t: the tensor-core layouts from fp_pack_pattention_weights (bf16 with K % 64 == 0 and
 *   D_out % 64 == 0; NULL otherwise, and every other shape or fp32 runs on CUDA cores).
 * fp_pack_pattention_weights is fp_pack_weights with separate widths: w_gu holds 2 * Np * K elements
 * (with k_up NULL the gate rows fill both halves of each packed block), v_t ceil(D_out / 256) * 256 * Np.
 */
FP_API int fp_pack_pattention_weights(const void* k_gate, const void* k_up, const void* v, int dtype, int Np,
                                      int K, int D_out, void* w_gu, void* v_t, void* stream);
FP_API size_t fp_pattention_workspace_size(int dtype, int64_t M, int K, int Np, int D_out, int n_active);
FP_API int fp_pattention_fwd(const void* x, int64_t M, int K, int Np, int D_out, int dtype, const void* k_gate,
                             const void* k_up, const void* v, const void* w_gu, const void* v_t,
                             const int32_t* active, int n_active, int activation, void* y, void* workspace,
                             size_t workspace_bytes, void* stream);

/*
 * SwiGLU of two pre-activation tensors, h = silu(g) * u (n elements, fp32 arithmetic, `dtype` in and
 * out): the forward of triton_fused_swiglu / TritonFusedSwiGLUFunction (pattention_triton.py:30-47,
 * :79-104).  Its backward is fp_swiglu_bwd.
 */
FP_API int fp_swiglu_fwd(const void* g, const void* u, int dtype, int64_t n, void* h, void* stream);

/*
 * Teacher block energies of the offline router calibration (FovealPattentionMLP.calibrate_offline_svd,
 * foveal_pattention.py:205-218):
 *   energy[t, b] = mean_{j in block b} |silu(x_t . k_gate_j) * (x_t . k_up_j)| * vnorm[b]
 * over all NB blocks (the dense SwiGLU of the calibration tokens), computed by the gate/up tensor-core
 * kernel with an fp32 reduction in its epilogue instead of writing the activations.
 *   x [M, D] bf16; w_gu from fp_pack_weights; vnorm [NB] fp32 (Frobenius norms of the blocks of v);
 *   energy [M, NB] fp32.  bf16 only, D % 64 == 0.
 */
FP_API size_t fp_block_energy_workspace_size(int64_t M, int NB);
FP_API int fp_block_energy(const void* x, int64_t M, int D, int NB, int dtype, const void* w_gu,
                           const float* vnorm, float* energy, void* workspace, size_t workspace_bytes,
                           void* stream);

/*
 * Fused SwiGLU backward of the active-set contraction (TritonFusedSwiGLUFunction.backward,
 * pattention_triton.py:49-96): for n elements of the gate / up pre-activations g, u and the upstream
 * gradient dout, dg = dout * u * silu'(g), du = dout * silu(g), and (optional, h may be NULL) the
 * activation h = silu(g) * u; fp32 arithmetic, all tensors in `dtype`.
 */
FP_API int fp_swiglu_bwd(const void* dout, const void* g, const void* u, int dtype, int64_t n, void* dg, void* du,
                         void* h, void* stream);

/*
 * Allocation-free token-routed forward (no counterpart in the reference).  Same arguments and result
 * as fp_pattention_token_fwd, without the workspace: it runs in a FP_NOALLOC_SCRATCH_BYTES scratch
 * array that the library keeps on each GPU it is loaded on, so callers that cannot allocate device
 * memory per call (plugin interfaces that only pass input/output pointers, serving loops with a
 * device-memory budget fixed at start-up) can still run the layer.  Calls needing more scratch than
 * the array holds (large batches; sized for decode-step batches) return FP_ERR_WORKSPACE.  All calls
 * on a device share the array: calls that overlap on the GPU race, so serialise them.  The first call
 * on a device looks up the array's address; make it before any stream capture.  The bounded-wait
 * error word of a call lives in the array: read it with fp_noalloc_device_error before the next
 * no-alloc call on that device (which clears it).
 */
#define FP_NOALLOC_SCRATCH_BYTES (16u << 20)
FP_API int fp_pattention_token_fwd_noalloc(const void* x, int64_t M, int D, int NB, int dtype,
                                           const void* k_gate, const void* k_up, const void* v, const void* w_gu,
                                           const void* v_t, const void* q_proj, const void* block_keys,
                                           const void* out_proj, int base_blocks, float top_p, int min_remote,
                                           int max_remote, float temperature, int additive, int block_stride,
                                           int block_offset, void* y, int y_f32, int32_t* remote_indices,
                                           int32_t* remote_counts, float* scores, void* stream);

/*
 * Device error word of the last fp_pattention_token_fwd_noalloc call on the current device (no
 * counterpart in the reference): synchronizes `stream`, returns FP_OK, FP_ERR_TIMEOUT (a bounded wait
 * of that call ran out, so its outputs are incomplete) or FP_ERR_CUDA, writes the raw code to *code and
 * clears the word, like fp_device_error on a caller's workspace.  Allocates nothing.
 */
FP_API int fp_noalloc_device_error(void* stream, int* code);

/* ------------------------------------------------------------------------------------------------
 * Layers that share the 16-D router but contract over the UNION of the blocks a call's tokens
 * selected: BlockSparseLinear (foveal_indexer/block_matmul.py:129-282) and FovealTokenformerLinear
 * (foveal_indexer/tokenformer.py:132-228).  A forward is: fp_param_blocks_16d (once per weight
 * update) -> fp_cosine_block_scores -> fp_select_blocks (routes and/or the additive-stream context
 * softmax(S) . v_blocks with temperature 1) or fp_select_remote_top_p -> fp_union_blocks ->
 * fp_block_sparse_linear_fwd or fp_tokenformer_fwd.  The union count stays on the device: no call of
 * the sequence synchronizes the host.
 * ------------------------------------------------------------------------------------------------ */

/*
 * Pooled 16-D key and value of every 64-row block of a parameter matrix P [N, D] (N % 64 == 0):
 *   k_blocks[b] = normalize(mean_{rows r of b} rms_norm(P[r] . k_proj^T))   fp32 [N / 64, 16]
 *   v_blocks[b] = mean_{rows r of b} P[r] . v_proj^T                        fp32 [N / 64, 16]
 * Replaces FovealIndexer.compute_kv_blocks_16d (core.py:225-252; Tokenformer's parameter keys,
 * tokenformer.py:150-155) and BlockSparseLinear.get_block_keys_and_values (block_matmul.py:107-127).
 * k_proj, v_proj [16, D] in `dtype`.
 */
FP_API int fp_param_blocks_16d(const void* P, const void* k_proj, const void* v_proj, int dtype, int64_t N, int D,
                               float* k_blocks, float* v_blocks, void* stream);

/*
 * Cosine block scores (FovealIndexer.compute_query_16d core.py:214-223, then compute_block_scores
 * core.py:254-266):  scores[m, b] = normalize(rms_norm(x[m] . q_proj^T)) . normalize(k_blocks[b]) / 4
 * x [M, D], q_proj [16, D] in `dtype`; k_blocks [NB, 16] fp32; scores [M, NB] fp32; q16 (optional)
 * [M, 16] fp32 receives rms_norm(x . q_proj^T).  D % 8 == 0, NB <= 1024.
 */
FP_API int fp_cosine_block_scores(const void* x, const void* q_proj, const float* k_blocks, int dtype, int64_t M,
                                  int D, int NB, float* scores, float* q16, void* stream);

/*
 * BlockSparseLinear's inference selection (block_matmul.py:185-201): per token, softmax over the
 * remote columns [base, NB) of scores [M, NB] only, and the first
 * count = min(#(cumsum < top_p) + 1, max_remote) block ids by descending probability (ties to the
 * lower id).  remote_indices [M, capacity] int32 receives absolute block ids; remote_counts [M] int32
 * the count, which (as in the reference) may exceed the NB - base available blocks by one when the
 * mass never reaches top_p; consumers read min(count, capacity) ids.  stats as in fp_select_blocks.
 */
FP_API int fp_select_remote_top_p(const float* scores, int64_t M, int NB, int base, float top_p, int max_remote,
                                  int capacity, int32_t* remote_indices, int32_t* remote_counts, float* stats,
                                  void* stream);

/*
 * Union of the selected blocks: blocks[0..n) = ascending ids of [0, base) and of every
 * remote_indices[m, i] with i < min(remote_counts[m], capacity); blocks[n..NB) = the other ids
 * ascending; *n_active = n (device int32).  block_matmul.py:206-217 (torch.where of the active mask),
 * tokenformer.py:171-181 (torch.unique after the base blocks).  NB <= 8192.
 */
FP_API int fp_union_blocks(const int32_t* remote_indices, const int32_t* remote_counts, int64_t M, int capacity,
                           int NB, int base, int32_t* blocks, int32_t* n_active, void* stream);

/* Workspace bytes of fp_block_sparse_linear_fwd (max_active as there). */
FP_API size_t fp_block_sparse_linear_workspace_size(int dtype, int64_t M, int D_in, int out_features, int max_active);

/*
 * BlockSparseLinear contraction (block_matmul.py:233-254):
 *   out[m, c] = x[m] . weight[c] + bias[c] + ctx16[m] . out_proj[c]   for c in an active block
 *   out[m, c] = ctx16[m] . out_proj[c]                                for c in an inactive block
 * (the ctx16 terms only when ctx16 != NULL; otherwise inactive columns are 0).  x [M, D_in],
 * weight [out_features, D_in], bias [out_features] (optional), out_proj [out_features, 16] and out
 * [M, out_features] in `dtype`; blocks / n_active from fp_union_blocks; ctx16 [M, 16] fp32.
 * out_features % 64 == 0.  bf16 with D_in % 64 == 0 runs on the tensor cores (tcgen05), everything
 * else on CUDA cores.  max_active: an upper bound of *n_active known on the host (e.g. base +
 * M * capacity; <= 0 = out_features / 64), from which batches of few tokens size a split of the
 * contraction.  Workspace: fp_block_sparse_linear_workspace_size bytes, at least
 * FP_VARIANT_WORKSPACE_MIN (device error word).
 */
#define FP_VARIANT_WORKSPACE_MIN 256u
FP_API int fp_block_sparse_linear_fwd(const void* x, int64_t M, int D_in, const void* weight, const void* bias,
                                      int out_features, int dtype, const int32_t* blocks, const int32_t* n_active,
                                      int max_active, const float* ctx16, const void* out_proj, void* out,
                                      void* workspace, size_t workspace_bytes, void* stream);

/*
 * 64 x 64 blocked copy of a row-major bf16 weight [rows, cols] (rows, cols multiples of 64): tile
 * (kb, j) = weight rows [j*64, +64) x columns [kb*64, +64), stored as one contiguous 8 KB run of 64-element
 * rows at tile index kb * (rows / 64) + j.  out: rows * cols bf16, 16-byte aligned.  The tensor-core
 * contraction of fp_block_sparse_linear_blocked_fwd then reads one selected block at one k-block as one
 * 8 KB run, and four consecutive blocks as one 32 KB run, instead of 64 row pieces of 128 bytes.
 */
FP_API int fp_pack_blocked_weight(const void* weight, int rows, int cols, void* out, void* stream);

/*
 * fp_block_sparse_linear_fwd with the weight's blocked copy (fp_pack_blocked_weight of weight
 * [out_features, D_in]; bf16, D_in % 64 == 0) as the tensor cores' operand.  weight stays required (the
 * CUDA-core path for shapes the tensor path does not tile reads it); weight_blocked == NULL is
 * fp_block_sparse_linear_fwd.  Same workspace.
 */
FP_API int fp_block_sparse_linear_blocked_fwd(const void* x, int64_t M, int D_in, const void* weight,
                                              const void* weight_blocked, const void* bias, int out_features,
                                              int dtype, const int32_t* blocks, const int32_t* n_active,
                                              int max_active, const float* ctx16, const void* out_proj, void* out,
                                              void* workspace, size_t workspace_bytes, void* stream);

/*
 * FovealTokenformerLinear contraction over the active parameter tokens (tokenformer.py:183-203):
 *   s = x . K_act^T,  p = softmax(s / sqrt(D_in)) (activation 0) or gelu(normalize(s)) (activation 1),
 *   out = p . V_act + ctx16 . out_proj^T
 * where K_act / V_act are the rows of k_param [Np, D_in] / v_param [Np, D_out] of the blocks
 * blocks[0..n_active) in that order.  v_param_t [D_out, Np] = v_param transposed (fp_transpose; the
 * tensor-core operand, may be NULL for fp32).  ctx16 optional.  bf16 with D_in % 64 == 0 and
 * D_out % 64 == 0 runs on the tensor cores, everything else on CUDA cores.
 */
FP_API size_t fp_tokenformer_workspace_size(int dtype, int64_t M, int num_param_tokens);
FP_API int fp_tokenformer_fwd(const void* x, int64_t M, int D_in, const void* k_param, const void* v_param,
                              const void* v_param_t, int num_param_tokens, int D_out, int dtype, int activation,
                              const int32_t* blocks, const int32_t* n_active, const float* ctx16,
                              const void* out_proj, void* out, void* workspace, size_t workspace_bytes,
                              void* stream);

/* dst [cols, rows] = src [rows, cols] transposed, in `dtype`. */
FP_API int fp_transpose(const void* src, int64_t rows, int64_t cols, int dtype, void* dst, void* stream);

/*
 * Measurement hook (no counterpart in the reference): for the calling host thread, the forward entry
 * points record events[i] (cudaEvent_t handles) on their stream at stage boundaries:
 *   fp_pattention_token_fwd:  0 start, 1 and 2 routed (scores, selection, block lists and H clears are
 *                             one projection kernel and one routing kernel), 3 gate/up kernel done,
 *                             4 down kernel done
 *   fp_pattention_pooled_fwd: 0 start, 1 gate/up kernel done, 2 down kernel done
 * Boundaries past n_events are not recorded.  events = NULL or n_events = 0 turns the hook off.
 */
FP_API int fp_set_stage_events(void* const* events, int n_events);

/*
 * Reads (and clears) the device error word of a workspace after synchronizing `stream`.  Returns
 * FP_OK, FP_ERR_TIMEOUT (a bounded wait ran out) or FP_ERR_CUDA; *code receives the raw device code.
 */
FP_API int fp_device_error(void* workspace, void* stream, int* code);

#ifdef __cplusplus
}
#endif

#endif /* FOVEAL_PATTENTION_H_ */
