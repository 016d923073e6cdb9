// Allocation-free variant of the token-routed forward.
//
// fp_pattention_token_fwd needs a caller-provided workspace (scores, routes, block lists, the masked
// activations H).  Some callers cannot allocate device memory at the point where they run the layer:
// plugin interfaces that hand the layer only its input and output pointers, or serving loops whose
// device-memory budget is fixed at start-up and forbid cudaMalloc/cudaFree afterwards.  For them,
// fp_pattention_token_fwd_noalloc uses a scratch area that lives in this library as a file-scope
// __device__ array, sized for small batches (decode steps).  Nothing is allocated per call.
//
// Limits and sharing rules:
//   * FP_NOALLOC_SCRATCH_BYTES (16 MiB) is reserved on every GPU that loads this library, until the
//     process exits.  Calls whose workspace would exceed it return FP_ERR_WORKSPACE.
//   * All calls on a device share the one array and it keeps the previous call's contents.  The
//     forward clears everything that must start at zero (error word, block counts, H, split-K
//     accumulators) at the start of each call.  Calls that overlap on the GPU (different streams
//     or threads without ordering between them) race on the array: serialise them.
//   * The first call on a device looks up the array's device address (cudaGetSymbolAddress with
//     that device current) and caches it; make that first call before any stream capture.
//   * The bounded-wait error word of a call lives at the start of the shared array (the workspace
//     layout of the token forward puts it at offset 0).  fp_noalloc_device_error reads and clears it;
//     read it before the next no-alloc call on the device, which clears it again.
#include "fp_internal.cuh"

#include <mutex>

namespace fp {
namespace {

constexpr size_t kNoAllocScratchBytes = FP_NOALLOC_SCRATCH_BYTES;
static_assert(kNoAllocScratchBytes % 256 == 0, "scratch size must keep 256-byte alignment");
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_dev_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (host code must not use the symbol
// itself as a pointer: on the host it is only a stand-in for the device object).
int scratch_on_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FP_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return FP_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_dev_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return FP_ERR_CUDA;
    g_scratch_dev_ptr[dev] = p;
  }
  *out = g_scratch_dev_ptr[dev];
  return FP_OK;
}

}  // namespace
}  // namespace fp

extern "C" {

int fp_pattention_token_fwd_noalloc(const void* x, int64_t M, int D, int NB, int dtype, const void* k_gate,
                                    const void* k_up, const void* v, const void* w_gu, const void* v_t,
                                    const void* q_proj, const void* block_keys, const void* out_proj,
                                    int base_blocks, float top_p, int min_remote, int max_remote,
                                    float temperature, int additive, int block_stride, int block_offset, void* y,
                                    int y_f32, int32_t* remote_indices, int32_t* remote_counts, float* scores,
                                    void* stream) {
  if (block_stride < 1) return FP_ERR_INVALID_ARG;
  const size_t need = fp::token_workspace_size_min(dtype, M, D, NB, base_blocks, max_remote, block_stride);
  if (need > fp::kNoAllocScratchBytes) return FP_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int rc = fp::scratch_on_current_device(&scratch);
  if (rc != FP_OK) return rc;
  return fp_pattention_token_fwd(x, M, D, NB, dtype, k_gate, k_up, v, w_gu, v_t, q_proj, block_keys, out_proj,
                                 base_blocks, top_p, min_remote, max_remote, temperature, additive, block_stride,
                                 block_offset, y, y_f32, remote_indices, remote_counts, scores, scratch,
                                 fp::kNoAllocScratchBytes, stream);
}

int fp_noalloc_device_error(void* stream, int* code) {
  void* scratch = nullptr;
  const int rc = fp::scratch_on_current_device(&scratch);
  if (rc != FP_OK) return rc;
  return fp_device_error(scratch, stream, code);  // error word at offset 0 of the token-forward layout
}

}  // extern "C"
