// Column-block W2A16 g128 GEMV kernels (sm_100a, CUDA cores, dp2a inner product).
//
//  gemv_kernel: the reference's moe_gemv_int2_tab (gemv/moe_gemv_int2_tab.py:23-85):
//               c[r, n] = (w_r if mul) * sum_k deq(W_{ids[r]})[k, n] * a[r / top_k, k]
// (the whole decode layer runs in the fused kernel of w2a16_layer.cu).
//
// One CTA = one block of 128 output columns (32 lanes x 4 columns, one 16-byte load per word row) for one
// routed row. Its warps split the K groups; each lane streams 8 word rows (one group) per step with
// 16-byte loads, with the next group's loads in flight while the current one is reduced. Cross-warp sums
// go through shared memory in a fixed order, so results are deterministic.
#include "w2a16_common.cuh"
#include "w2a16_kernels.h"

namespace w2a16 {

struct GemvParams {
  const void* a;          // activations: bf16 [*, K]
  int64_t stride_am;      // elements
  ExpertMap map;
  const int32_t* ids;     // [R]
  const float* topk_w;    // [R]
  void* out;              // bf16 [R, N]
  int64_t stride_om;      // elements
  int R, N, K, top_k;
  int64_t stride_ww;      // words per K/16 row
  int64_t stride_sg;      // scale elements per group row
  int64_t stride_zg;      // zero bytes per group row
  int mul_routed_weight;
  int scale_bf16;
  unsigned* err;
};

__device__ __forceinline__ void load_group_words(const uint32_t* __restrict__ wp, int64_t stride_ww, uint4 (&W)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) W[i] = __ldg(reinterpret_cast<const uint4*>(wp + (int64_t)i * stride_ww));
}

// One lane-task: 4 columns x 1 group. Returns the group's fp32 contribution per column.
__device__ __forceinline__ void group_task(const uint4 (&W)[8], const uint32_t* __restrict__ xpairs, int g,
                                           int m64x, float scl, const float (&s)[4], uint32_t zbyte,
                                           bool has_z, float (&colacc)[4], float wmul) {
  int acc[4][4];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[c][j] = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint4* xp = reinterpret_cast<const uint4*>(xpairs + (g * 8 + i) * kXRegs);
    const uint4 xa = xp[0], xb = xp[1];
    const uint32_t xr[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
    word_dot(W[i].x, xr, acc[0]);
    word_dot(W[i].y, xr, acc[1]);
    word_dot(W[i].z, xr, acc[2]);
    word_dot(W[i].w, xr, acc[3]);
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int zp = has_z ? (int)((zbyte >> (2 * c)) & 3u) : 2;
    const int T = combine_classes(acc[c]) + zp * m64x;
    colacc[c] = fmaf((float)T, s[c] * scl * wmul, colacc[c]);
  }
}

__global__ void __launch_bounds__(512) gemv_kernel(GemvParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int nwarps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.K / kGroup;
  XTable tab;
  tab.pairs = reinterpret_cast<uint32_t*>(smem);
  tab.m64x = reinterpret_cast<int*>(smem + (size_t)(p.K / 16) * kXRegs * 4);
  tab.scl = reinterpret_cast<float*>(tab.m64x + G);
  float* red = reinterpret_cast<float*>(tab.scl + G);   // [nwarps][128]

  const int q = blockIdx.x * 32 + lane;                  // column quad of this lane
  const bool lane_active = q * 4 < p.N;
  float colacc[4] = {0.f, 0.f, 0.f, 0.f};
  const bool sbf = p.scale_bf16 != 0;
  const bool has_z = p.map.has_zeros != 0;

  const int r = blockIdx.y;
  const int e = p.ids[r];
  const uint32_t* wbase;
  const char* sbase;
  const uint8_t* zbase = nullptr;
  const bool ok = p.map.resolve(e, wbase, sbase, zbase, p.err);   // masked row: contributes zero
  if (ok) {
    const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(p.a) + (int64_t)(r / p.top_k) * p.stride_am;
    for (int g = warp; g < G; g += nwarps) prep_group_warp<__nv_bfloat16>(src + g * kGroup, g, tab, lane);
    __syncthreads();
    const float wmul = p.mul_routed_weight ? p.topk_w[r] : 1.f;
    if (lane_active) {
      const uint32_t* wq = wbase + 4 * q;
      uint4 Wc[8], Wn[8];
      int g = warp;
      if (g < G) load_group_words(wq + (int64_t)(8 * g) * p.stride_ww, p.stride_ww, Wc);
      for (; g < G; g += nwarps) {
        const int gn = g + nwarps;
        if (gn < G) load_group_words(wq + (int64_t)(8 * gn) * p.stride_ww, p.stride_ww, Wn);
        float s[4];
        load_scale4(sbase, (int64_t)g * p.stride_sg + 4 * q, sbf, s);
        const uint32_t zb = has_z ? (uint32_t)zbase[(int64_t)g * p.stride_zg + q] : 0u;
        group_task(Wc, tab.pairs, g, tab.m64x[g], tab.scl[g], s, zb, has_z, colacc, wmul);
#pragma unroll
        for (int i = 0; i < 8; ++i) Wc[i] = Wn[i];
      }
    }
  }

  // cross-warp reduction in a fixed order
  __syncthreads();
#pragma unroll
  for (int c = 0; c < 4; ++c) red[warp * 128 + lane * 4 + c] = colacc[c];
  __syncthreads();
  for (int t = threadIdx.x; t < 128; t += blockDim.x) {
    float v = 0.f;
    for (int w = 0; w < nwarps; ++w) v += red[w * 128 + t];
    const int n = blockIdx.x * 128 + t;
    if (n < p.N) {
      __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(p.out) + (int64_t)r * p.stride_om;
      op[n] = __float2bfloat16(ok ? v : 0.f);
    }
  }
}

static size_t gemv_smem_bytes(int K, int nwarps) {
  const int G = K / kGroup;
  return (size_t)(K / 16) * kXRegs * 4 + (size_t)G * 8 + (size_t)nwarps * 128 * 4;
}

static int pick_warps(int K) {
  const int G = K / kGroup;
  return G < 16 ? G : 16;
}

static int launch_gemv(const GemvParams& p, dim3 grid, cudaStream_t stream) {
  const int nw = pick_warps(p.K);
  const size_t smem = gemv_smem_bytes(p.K, nw);
  auto kern = gemv_kernel;
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return kErrLaunch;
  }
  kern<<<grid, nw * 32, smem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

// ----------------------------------------------------------------------------- host entry points
int gemv_plain(const GemvArgs& g) {
  if (g.R <= 0) return kOk;
  if (g.K <= 0 || g.K % kGroup != 0 || g.N <= 0 || g.N % 4 != 0) return kErrShape;
  if (g.stride_ww % 4 != 0 || g.stride_sg % 4 != 0 || g.stride_ww < g.N || g.stride_sg < g.N) return kErrAlign;
  if (g.top_k <= 0 || !g.a || !g.ids || !g.out || (g.mul_routed_weight && !g.topk_w)) return kErrArg;
  GemvParams p{};
  p.a = g.a; p.stride_am = g.stride_am; p.map = g.map; p.ids = g.ids; p.topk_w = g.topk_w;
  p.out = g.out; p.stride_om = g.stride_om; p.R = g.R; p.N = g.N; p.K = g.K; p.top_k = g.top_k;
  p.stride_ww = g.stride_ww; p.stride_sg = g.stride_sg; p.stride_zg = g.stride_zg;
  p.mul_routed_weight = g.mul_routed_weight; p.scale_bf16 = g.scale_bf16;
  p.err = g.err;
  dim3 grid((g.N + 127) / 128, g.R);
  return launch_gemv(p, grid, g.stream);
}

}  // namespace w2a16
