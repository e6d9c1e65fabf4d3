// extern "C" entry points declared in include/w2a16_moe.h. Argument checking, expert-map
// construction and dispatch only; the kernels live in the other translation units.
#include "../../include/w2a16_moe.h"
#include "w2a16_kernels.h"

using namespace w2a16;

namespace {

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

ExpertMap table_map(const int64_t* wtab, const int64_t* stab, const int64_t* ztab, int E) {
  ExpertMap m{};
  m.wtab = wtab; m.stab = stab; m.ztab = ztab; m.E = E; m.has_zeros = ztab != nullptr;
  return m;
}

ExpertMap slot_map(const int32_t* slots, int E, int S, const void* cb, int64_t cs, const void* sb, int64_t ss,
                   const void* zb, int64_t zs) {
  ExpertMap m{};
  m.slots = slots; m.E = E; m.S = S;
  m.wbase = static_cast<const char*>(cb); m.wstride = cs;
  m.sbase = static_cast<const char*>(sb); m.sstride = ss;
  m.zbase = static_cast<const char*>(zb); m.zstride = zs;
  m.has_zeros = zb != nullptr;
  return m;
}

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

const char* w2a16_version(void) { return "w2a16_moe 0.1 sm_100a"; }

const char* w2a16_status_string(int s) {
  switch (s) {
    case W2A16_OK: return "ok";
    case W2A16_ERR_SHAPE: return "unsupported shape";
    case W2A16_ERR_ALIGN: return "misaligned stride or base address";
    case W2A16_ERR_LAUNCH: return "CUDA launch failed";
    case W2A16_ERR_ARG: return "invalid argument";
    case W2A16_ERR_WORKSPACE: return "workspace missing or too small";
    case W2A16_ERR_DEVICE: return "no usable sm_100 device";
    case W2A16_ERR_MEMORY: return "no memory for another arena chunk";
    default: return "unknown status";
  }
}

int w2a16_moe_gemv_tab(const void* a, int64_t stride_am, const int64_t* wtab, const int64_t* stab,
                       const int64_t* ztab, int num_experts, const int32_t* topk_ids, const float* topk_w,
                       void* c, int64_t stride_cm, int R, int N, int K, int64_t stride_ww, int64_t stride_sg,
                       int64_t stride_zg, int top_k, int mul_routed_weight, int scale_bf16, unsigned int* err,
                       void* stream) {
  if (!wtab || !stab || num_experts <= 0) return W2A16_ERR_ARG;
  GemvArgs g{};
  g.a = a; g.stride_am = stride_am; g.map = table_map(wtab, stab, ztab, num_experts);
  g.ids = topk_ids; g.topk_w = topk_w; g.out = c; g.stride_om = stride_cm;
  g.R = R; g.N = N; g.K = K; g.top_k = top_k;
  g.stride_ww = stride_ww; g.stride_sg = stride_sg; g.stride_zg = stride_zg;
  g.mul_routed_weight = mul_routed_weight; g.scale_bf16 = scale_bf16; g.err = err; g.stream = as_stream(stream);
  if (ztab && (stride_zg < N / 4)) return W2A16_ERR_ALIGN;
  return gemv_plain(g);
}

int w2a16_moe_gemv_slots(const void* a, int64_t stride_am, const int32_t* slots, int num_experts, int num_slots,
                         const void* codes_base, int64_t codes_slot_bytes, const void* scales_base,
                         int64_t scales_slot_bytes, const void* zeros_base, int64_t zeros_slot_bytes,
                         const int32_t* topk_ids, const float* topk_w, void* c, int64_t stride_cm, int R, int N,
                         int K, int top_k, int mul_routed_weight, int scale_bf16, unsigned int* err, void* stream) {
  if (!slots || num_experts <= 0 || num_slots <= 0 || !codes_base || !scales_base) return W2A16_ERR_ARG;
  if (!a16(codes_base) || !a16(scales_base) || codes_slot_bytes % 16 || scales_slot_bytes % 16) return W2A16_ERR_ALIGN;
  GemvArgs g{};
  g.a = a; g.stride_am = stride_am;
  g.map = slot_map(slots, num_experts, num_slots, codes_base, codes_slot_bytes, scales_base, scales_slot_bytes, zeros_base,
                   zeros_slot_bytes);
  g.ids = topk_ids; g.topk_w = topk_w; g.out = c; g.stride_om = stride_cm;
  g.R = R; g.N = N; g.K = K; g.top_k = top_k;
  g.stride_ww = N; g.stride_sg = N; g.stride_zg = N / 4;
  g.mul_routed_weight = mul_routed_weight; g.scale_bf16 = scale_bf16; g.err = err; g.stream = as_stream(stream);
  return gemv_plain(g);
}

size_t w2a16_moe_layer_workspace_bytes(int M, int H, int I, int top_k) {
  return layer_workspace_bytes(M, H, I, top_k);
}

size_t w2a16_moe_layer_workspace_bytes_batched(int M, int H, int I, int top_k) {
  const size_t a = layer_workspace_bytes(M, H, I, top_k);
  if (M < kGroupedMinTokens) return a;
  const size_t b = grouped_workspace_bytes(M, H, I, top_k);
  return a > b ? a : b;
}

int w2a16_moe_decode_layer_tab(const void* x, int M, int H, int I, int top_k, const int32_t* topk_ids,
                               const float* topk_w, int num_experts, const int64_t* wtab13, const int64_t* stab13,
                               const int64_t* ztab13, const int64_t* wtab2, const int64_t* stab2,
                               const int64_t* ztab2, int scale_bf16, float routed_scaling_factor, void* y,
                               void* workspace, size_t workspace_bytes, unsigned int* err, void* stream) {
  if (!wtab13 || !stab13 || !wtab2 || !stab2 || num_experts <= 0) return W2A16_ERR_ARG;
  if ((ztab13 == nullptr) != (ztab2 == nullptr)) return W2A16_ERR_ARG;
  LayerArgs a{};
  a.x = x; a.M = M; a.H = H; a.I = I; a.top_k = top_k; a.ids = topk_ids; a.topk_w = topk_w;
  a.map13 = table_map(wtab13, stab13, ztab13, num_experts);
  a.map2 = table_map(wtab2, stab2, ztab2, num_experts);
  a.scale_bf16 = scale_bf16; a.routed_scaling = routed_scaling_factor; a.y = y;
  a.workspace = workspace; a.workspace_bytes = workspace_bytes; a.err = err; a.stream = as_stream(stream);
  return decode_layer_fused(a);
}

int w2a16_moe_decode_layer_slots_ex(const void* x, int M, int H, int I, int top_k, const int32_t* topk_ids,
                                    const float* topk_w, const int32_t* slots, int num_experts, int num_slots,
                                    const void* codes13, int64_t codes13_slot_bytes, const void* scales13,
                                    int64_t scales13_slot_bytes, const void* zeros13, int64_t zeros13_slot_bytes,
                                    const void* codes2, int64_t codes2_slot_bytes, const void* scales2,
                                    int64_t scales2_slot_bytes, const void* zeros2, int64_t zeros2_slot_bytes,
                                    int scale_bf16, float routed_scaling_factor, void* y, void* workspace,
                                    size_t workspace_bytes, int path, unsigned int* err, void* stream) {
  if (!slots || num_experts <= 0 || num_slots <= 0 || !codes13 || !scales13 || !codes2 || !scales2)
    return W2A16_ERR_ARG;
  if (path != W2A16_PATH_AUTO && path != W2A16_PATH_PER_TOKEN && path != W2A16_PATH_BATCHED) return W2A16_ERR_ARG;
  if ((zeros13 == nullptr) != (zeros2 == nullptr)) return W2A16_ERR_ARG;
  if (!a16(codes13) || !a16(scales13) || !a16(codes2) || !a16(scales2)) return W2A16_ERR_ALIGN;
  if (codes13_slot_bytes % 16 || scales13_slot_bytes % 16 || codes2_slot_bytes % 16 || scales2_slot_bytes % 16)
    return W2A16_ERR_ALIGN;
  if (zeros13 && (!a16(zeros13) || !a16(zeros2) || zeros13_slot_bytes % 16 || zeros2_slot_bytes % 16))
    return W2A16_ERR_ALIGN;
  LayerArgs a{};
  a.x = x; a.M = M; a.H = H; a.I = I; a.top_k = top_k; a.ids = topk_ids; a.topk_w = topk_w;
  a.map13 = slot_map(slots, num_experts, num_slots, codes13, codes13_slot_bytes, scales13, scales13_slot_bytes,
                     zeros13, zeros13_slot_bytes);
  a.map2 = slot_map(slots, num_experts, num_slots, codes2, codes2_slot_bytes, scales2, scales2_slot_bytes, zeros2,
                    zeros2_slot_bytes);
  a.scale_bf16 = scale_bf16; a.routed_scaling = routed_scaling_factor; a.y = y;
  a.workspace = workspace; a.workspace_bytes = workspace_bytes; a.err = err; a.stream = as_stream(stream);
  // The batched path (experts grouped over the tokens, each streamed once, products on the tensor cores) by
  // token count: from W2A16_BATCHED_AUTO_TOKENS tokens in AUTO mode when the workspace holds its buffers, from
  // 16 tokens when asked for; otherwise the per-token fused layer.
  if (path == W2A16_PATH_BATCHED) {
    const int st = grouped_check(a);
    return st == kOk ? decode_layer_grouped(a) : st;
  }
  if (path == W2A16_PATH_AUTO && M >= W2A16_BATCHED_AUTO_TOKENS && grouped_check(a) == kOk) {
    const int st = decode_layer_grouped(a);
    if (st != kErrShape) return st;
  }
  return decode_layer_fused(a);
}

namespace {
PeerExchange exchange_of(const w2a16_exchange& e) {
  PeerExchange x{};
  x.peers = e.peer_bufs; x.tag_off = e.tag_offset; x.n_max = e.n_max; x.rank = e.rank; x.world = e.world;
  x.epoch = e.epoch; x.spin_limit = e.spin_limit;
  return x;
}
}  // namespace

int w2a16_moe_decode_layer_slots_ep(const void* x, int M, int H, int I, int top_k, const int32_t* topk_ids,
                                    const float* topk_w, const int32_t* slots, int num_experts, int num_slots,
                                    const void* codes13, int64_t codes13_slot_bytes, const void* scales13,
                                    int64_t scales13_slot_bytes, const void* zeros13, int64_t zeros13_slot_bytes,
                                    const void* codes2, int64_t codes2_slot_bytes, const void* scales2,
                                    int64_t scales2_slot_bytes, const void* zeros2, int64_t zeros2_slot_bytes,
                                    int scale_bf16, float routed_scaling_factor, void* y, void* workspace,
                                    size_t workspace_bytes, int x_from_peers, int y_to_peers,
                                    const w2a16_exchange* exchange, unsigned int* err, void* stream) {
  if (!slots || num_experts <= 0 || num_slots <= 0 || !codes13 || !scales13 || !codes2 || !scales2)
    return W2A16_ERR_ARG;
  if ((x_from_peers || y_to_peers) && !exchange) return W2A16_ERR_ARG;
  if ((zeros13 == nullptr) != (zeros2 == nullptr)) return W2A16_ERR_ARG;
  if (!a16(codes13) || !a16(scales13) || !a16(codes2) || !a16(scales2)) return W2A16_ERR_ALIGN;
  if (codes13_slot_bytes % 16 || scales13_slot_bytes % 16 || codes2_slot_bytes % 16 || scales2_slot_bytes % 16)
    return W2A16_ERR_ALIGN;
  if (zeros13 && (!a16(zeros13) || !a16(zeros2) || zeros13_slot_bytes % 16 || zeros2_slot_bytes % 16))
    return W2A16_ERR_ALIGN;
  const PeerExchange ex = exchange ? exchange_of(*exchange) : PeerExchange{};
  LayerArgs a{};
  a.x = x_from_peers ? nullptr : x; a.M = M; a.H = H; a.I = I; a.top_k = top_k; a.ids = topk_ids; a.topk_w = topk_w;
  a.map13 = slot_map(slots, num_experts, num_slots, codes13, codes13_slot_bytes, scales13, scales13_slot_bytes,
                     zeros13, zeros13_slot_bytes);
  a.map2 = slot_map(slots, num_experts, num_slots, codes2, codes2_slot_bytes, scales2, scales2_slot_bytes, zeros2,
                    zeros2_slot_bytes);
  a.scale_bf16 = scale_bf16; a.routed_scaling = routed_scaling_factor; a.y = y_to_peers ? nullptr : y;
  a.workspace = workspace; a.workspace_bytes = workspace_bytes; a.err = err; a.stream = as_stream(stream);
  a.xin = x_from_peers ? &ex : nullptr;
  a.yout = y_to_peers ? &ex : nullptr;
  return decode_layer_fused(a);                 // an exchange call is one per-token launch
}

int w2a16_moe_decode_layer_slots(const void* x, int M, int H, int I, int top_k, const int32_t* topk_ids,
                                 const float* topk_w, const int32_t* slots, int num_experts, int num_slots,
                                 const void* codes13, int64_t codes13_slot_bytes, const void* scales13,
                                 int64_t scales13_slot_bytes, const void* zeros13, int64_t zeros13_slot_bytes,
                                 const void* codes2, int64_t codes2_slot_bytes, const void* scales2,
                                 int64_t scales2_slot_bytes, const void* zeros2, int64_t zeros2_slot_bytes,
                                 int scale_bf16, float routed_scaling_factor, void* y, void* workspace,
                                 size_t workspace_bytes, unsigned int* err, void* stream) {
  return w2a16_moe_decode_layer_slots_ex(x, M, H, I, top_k, topk_ids, topk_w, slots, num_experts, num_slots, codes13,
                                         codes13_slot_bytes, scales13, scales13_slot_bytes, zeros13,
                                         zeros13_slot_bytes, codes2, codes2_slot_bytes, scales2, scales2_slot_bytes,
                                         zeros2, zeros2_slot_bytes, scale_bf16, routed_scaling_factor, y, workspace,
                                         workspace_bytes, W2A16_PATH_AUTO, err, stream);
}

int w2a16_to_word_ncontig(const void* src_u8, void* dst_i32, int E, int N, int K, void* stream) {
  return to_word_ncontig(src_u8, dst_i32, E, N, K, as_stream(stream));
}

int w2a16_gather_rows_tab(const int64_t* tab, const int32_t* ids, int n, void* out, int64_t row_bytes, void* stream) {
  return gather_rows_tab(tab, ids, n, out, row_bytes, as_stream(stream));
}

size_t w2a16_int8_workspace_bytes(int M, int K, int N) { return int8_workspace_bytes(M, K, N); }

int w2a16_allreduce_peers_bf16(const void* in, void* out, int n, int n_max, const uint64_t* peer_bufs,
                               size_t flag_offset, int rank, int world, unsigned int* epoch, unsigned int* err,
                               unsigned int spin_limit, void* stream) {
  return allreduce_peers_bf16(in, out, n, n_max, peer_bufs, flag_offset, rank, world, epoch, err, spin_limit,
                              as_stream(stream));
}

int w2a16_int8_gemv(const void* x, int64_t stride_xm, const int32_t* qweight, const void* scales, int group,
                    int zero, int M, int K, int N, void* y, int64_t stride_ym, void* workspace,
                    size_t workspace_bytes, void* stream) {
  Int8Args a{};
  a.x = x; a.stride_xm = stride_xm; a.qweight = qweight; a.scales = scales; a.group = group; a.zero = zero;
  a.M = M; a.K = K; a.N = N; a.y = y; a.stride_ym = stride_ym; a.stream = as_stream(stream);
  return int8_gemv(a, workspace, workspace_bytes);
}

int w2a16_int8_gemv_from_peers(const w2a16_exchange* exchange, const int32_t* qweight, const void* scales, int group,
                               int zero, int M, int K, int N, void* y, int64_t stride_ym, unsigned int* err,
                               void* stream) {
  if (!exchange) return W2A16_ERR_ARG;
  Int8Args a{};
  a.x = nullptr; a.stride_xm = K; a.qweight = qweight; a.scales = scales; a.group = group; a.zero = zero;
  a.M = M; a.K = K; a.N = N; a.y = y; a.stride_ym = stride_ym; a.stream = as_stream(stream);
  return int8_gemv_from_peers(a, exchange_of(*exchange), err);
}

}  // extern "C"
