// Decode-layer entry point that allocates nothing, for callers that cannot allocate device memory.
//
// Who needs it: a host that captures its decode step into a CUDA graph and reaches this call while the
// stream is being captured (cudaMalloc is not allowed during a global-mode capture), and serving
// processes whose device memory is fully reserved by their own pool at start-up (SGLang reserves its
// KV pool that way), where a late cudaMalloc fails or takes memory the pool counts on. Such callers can
// pass inputs and outputs they already own, but cannot provide the layer's workspace.
//
// So the workspace lives in a file-scope __device__ array of W2A16_NOALLOC_SCRATCH_BYTES bytes. Every GPU
// that loads this library holds that array until the process exits. Host code cannot use the array's
// name as a device address (on the host it is only a stand-in symbol); its device address is taken with
// cudaGetSymbolAddress, with the device current, on the first call made in each CUDA context (a device
// reset creates a new context, in which the array may sit elsewhere, so the address is looked up again).
#include <cudaTypedefs.h>
#include <mutex>

#include "../../include/w2a16_moe.h"
#include "w2a16_kernels.h"

namespace {

// Zero-initialised at module load. The layer kernels need their two barrier words equal on entry and
// leave them equal on exit, and their hand-off words tagged with no future epoch (zero qualifies); the rest
// of the array (the SiLU*mul activations and partial sums) is overwritten by every call.
__device__ __align__(256) unsigned char g_noalloc_scratch[W2A16_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};

// The driver's cuCtxGetCurrent through the runtime's entry-point query (the library links no driver library).
PFN_cuCtxGetCurrent_v4000 ctx_getter() {
  static PFN_cuCtxGetCurrent_v4000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<PFN_cuCtxGetCurrent_v4000>(nullptr);
    return reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f);
  }();
  return fn;
}

// Device address of g_noalloc_scratch in the calling thread's current device and context, looked up once
// per (device, context).
int scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return W2A16_ERR_DEVICE;
  const PFN_cuCtxGetCurrent_v4000 get = ctx_getter();
  if (get == nullptr) return W2A16_ERR_DEVICE;
  CUcontext ctx = nullptr;
  if (get(&ctx) != CUDA_SUCCESS) return W2A16_ERR_DEVICE;   // null before the thread's first CUDA call
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (ctx == nullptr || g_scratch_addr[dev] == nullptr || g_scratch_ctx[dev] != ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);   // (makes the primary context current)
    if (e != cudaSuccess || p == nullptr) return W2A16_ERR_DEVICE;
    if (ctx == nullptr && (get(&ctx) != CUDA_SUCCESS || ctx == nullptr)) return W2A16_ERR_DEVICE;
    g_scratch_addr[dev] = p;
    g_scratch_ctx[dev] = ctx;
  }
  *out = g_scratch_addr[dev];
  return W2A16_OK;
}

}  // namespace

extern "C" int w2a16_moe_decode_layer_slots_noalloc(
    const void* x, int M, int H, int I, int top_k, const int32_t* topk_ids, const float* topk_w,
    const int32_t* slots, int num_experts, int num_slots, const void* codes13, int64_t codes13_slot_bytes,
    const void* scales13, int64_t scales13_slot_bytes, const void* zeros13, int64_t zeros13_slot_bytes,
    const void* codes2, int64_t codes2_slot_bytes, const void* scales2, int64_t scales2_slot_bytes,
    const void* zeros2, int64_t zeros2_slot_bytes, int scale_bf16, float routed_scaling_factor, void* y,
    unsigned int* err, void* stream) {
  if (M < 0 || H <= 0 || I <= 0 || top_k <= 0) return W2A16_ERR_ARG;
  if (w2a16::layer_workspace_bytes(M, H, I, top_k) > (size_t)W2A16_NOALLOC_SCRATCH_BYTES)
    return W2A16_ERR_WORKSPACE;  // M * top_k * I too large for the fixed scratch array
  void* ws = nullptr;
  const int st = scratch_address(&ws);
  if (st != W2A16_OK) return st;
  // The same path choice as w2a16_moe_decode_layer_slots given this much workspace: per-token below
  // W2A16_BATCHED_AUTO_TOKENS tokens, batched from there on when its buffers fit the array.
  return w2a16_moe_decode_layer_slots_ex(x, M, H, I, top_k, topk_ids, topk_w, slots, num_experts, num_slots, codes13,
                                         codes13_slot_bytes, scales13, scales13_slot_bytes, zeros13,
                                         zeros13_slot_bytes, codes2, codes2_slot_bytes, scales2, scales2_slot_bytes,
                                         zeros2, zeros2_slot_bytes, scale_bf16, routed_scaling_factor, y, ws,
                                         (size_t)W2A16_NOALLOC_SCRATCH_BYTES, W2A16_PATH_AUTO, err, stream);
}
