// Decode MoE layer: gate_up GEMV + SiLU*mul, down GEMV * routed weight, sum over top-k
// (the composite of patches/ncontig_gemv.py:218-238).
#include "w2a16_kernels.h"

namespace w2a16 {

// Workspace layout (bytes): [0, 256): control words (error flags, counters); then h fp32 [R, I].
size_t layer_workspace_bytes(int M, int H, int I, int top_k) {
  (void)H;
  const size_t R = (size_t)M * (size_t)top_k;
  return 256 + R * (size_t)I * 4;
}

int decode_layer_two_pass(const LayerArgs& a) {
  if (a.M <= 0) return kOk;
  if (a.H % kGroup != 0 || a.I % kGroup != 0 || a.H % 4 != 0 || a.top_k <= 0) return kErrShape;
  if (!a.x || !a.ids || !a.topk_w || !a.y) return kErrArg;
  if (!a.workspace || a.workspace_bytes < layer_workspace_bytes(a.M, a.H, a.I, a.top_k)) return kErrWorkspace;
  const int R = a.M * a.top_k;
  float* h = reinterpret_cast<float*>(static_cast<char*>(a.workspace) + 256);

  GemvArgs g{};
  g.a = a.x; g.stride_am = a.H; g.map = a.map13; g.ids = a.ids; g.topk_w = a.topk_w;
  g.out = nullptr; g.stride_om = 0; g.R = R; g.N = 2 * a.I; g.K = a.H; g.top_k = a.top_k;
  g.stride_ww = 2 * a.I; g.stride_sg = 2 * a.I; g.stride_zg = (2 * a.I) / 4;
  g.mul_routed_weight = 0; g.scale_bf16 = a.scale_bf16; g.err = a.err; g.stream = a.stream;
  int st = gemv_gateup_silu(g, a.I, h, a.I);
  if (st != kOk) return st;

  GemvArgs d{};
  d.a = h; d.stride_am = a.I; d.map = a.map2; d.ids = a.ids; d.topk_w = a.topk_w;
  d.out = a.y; d.stride_om = a.H; d.R = R; d.N = a.H; d.K = a.I; d.top_k = a.top_k;
  d.stride_ww = a.H; d.stride_sg = a.H; d.stride_zg = a.H / 4;
  d.mul_routed_weight = 1; d.scale_bf16 = a.scale_bf16; d.err = a.err; d.stream = a.stream;
  return gemv_down_sum(d, a.M, a.routed_scaling);
}

int decode_layer_fused(const LayerArgs& a) { return decode_layer_two_pass(a); }

}  // namespace w2a16
