// Column-block W2A16 g128 GEMV kernels (sm_100a, CUDA cores, dp2a inner product).
//
//  * gemv_kernel<MODE_PLAIN>   : the reference's moe_gemv_int2_tab (gemv/moe_gemv_int2_tab.py:23-85):
//                                c[r, n] = (w_r if mul) * sum_k deq(W_{ids[r]})[k, n] * a[r / top_k, k]
//  * gemv_kernel<MODE_GATEUP>  : gate_up GEMV with SiLU(gate) * up fused (patches/ncontig_gemv.py:229-231)
//                                h[r, c] = silu(g_c) * u_c, gate = columns [0, I), up = [I, 2I), fp32
//  * gemv_kernel<MODE_DOWNSUM> : down GEMV times the routed weight, summed over the top-k rows of a
//                                token and scaled (patches/ncontig_gemv.py:232-237), bf16 [M, H]
//
// One CTA = one block of 128 output columns (32 lanes x 4 columns, one 16-byte load per word row)
// for one row (PLAIN / GATEUP) or one token (DOWNSUM). Its warps split the K groups; each lane
// streams 8 word rows (one group) per step with 16-byte loads, with the next group's loads in flight
// while the current one is reduced. Cross-warp sums go through shared memory in a fixed order, so
// results are deterministic.
#include "w2a16_common.cuh"
#include "w2a16_kernels.h"

namespace w2a16 {

enum Mode : int { MODE_PLAIN = 0, MODE_GATEUP = 1, MODE_DOWNSUM = 2 };

struct GemvParams {
  const void* a;          // activations: bf16 [*, K] (PLAIN/GATEUP) or fp32 [R, K] (DOWNSUM)
  int64_t stride_am;      // elements
  ExpertMap map;
  const int32_t* ids;     // [R]
  const float* topk_w;    // [R]
  void* out;              // PLAIN: bf16 [R, N]; GATEUP: fp32 [R, I]; DOWNSUM: bf16 [M, N]
  int64_t stride_om;      // elements
  int R, N, K, top_k;
  int64_t stride_ww;      // words per K/16 row
  int64_t stride_sg;      // scale elements per group row
  int64_t stride_zg;      // zero bytes per group row
  int I;                  // GATEUP: intermediate size (gate at [0, I), up at [I, 2I))
  int mul_routed_weight;
  int scale_bf16;
  float routed_scaling;
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

template <int MODE, typename AT>
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

  // column quad of this lane
  int q;           // quad index within the weight matrix
  int out_col;     // first output column of the quad (PLAIN/DOWNSUM) or h column (GATEUP)
  if (MODE == MODE_GATEUP) {
    const int hq = blockIdx.x * 16 + (lane & 15);           // h quad
    out_col = hq * 4;
    q = (lane < 16) ? hq : (p.I / 4 + hq);
  } else {
    q = blockIdx.x * 32 + lane;
    out_col = q * 4;
  }
  const int ncols_valid = (MODE == MODE_GATEUP) ? p.I : p.N;
  const bool lane_active = out_col < ncols_valid;

  float colacc[4] = {0.f, 0.f, 0.f, 0.f};
  const bool sbf = p.scale_bf16 != 0;
  const bool has_z = p.map.has_zeros != 0;

  const int nrows = (MODE == MODE_DOWNSUM) ? p.top_k : 1;
  bool any_row = false;
  for (int j = 0; j < nrows; ++j) {
    const int r = (MODE == MODE_DOWNSUM) ? blockIdx.y * p.top_k + j : blockIdx.y;
    const int e = p.ids[r];
    const uint32_t* wbase;
    const char* sbase;
    const uint8_t* zbase = nullptr;
    const bool ok = p.map.resolve(e, wbase, sbase, zbase, p.err);
    if (!ok) continue;                                       // masked row: contributes zero
    any_row = true;
    const int arow = (MODE == MODE_DOWNSUM) ? r : r / p.top_k;
    const AT* src = reinterpret_cast<const AT*>(p.a) + (int64_t)arow * p.stride_am;
    __syncthreads();                                         // previous row's table no longer read
    for (int g = warp; g < G; g += nwarps) prep_group_warp<AT>(src + g * kGroup, g, tab, lane);
    __syncthreads();
    const float wmul = (MODE == MODE_DOWNSUM) ? p.topk_w[r]
                       : ((MODE == MODE_PLAIN && p.mul_routed_weight) ? p.topk_w[r] : 1.f);
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
    if (MODE == MODE_GATEUP) {
      // t < 64: gate columns of this block, t >= 64: up columns (lane 16.. wrote them)
      if (t < 64) {
        const float gte = v;
        const float up = [&] { float u = 0.f; for (int w = 0; w < nwarps; ++w) u += red[w * 128 + 64 + t]; return u; }();
        const int c = blockIdx.x * 64 + t;
        if (c < p.I) {
          float* hp = reinterpret_cast<float*>(p.out) + (int64_t)blockIdx.y * p.stride_om;
          hp[c] = any_row ? silu(gte) * up : 0.f;
        }
      }
    } else {
      const int n = blockIdx.x * 128 + t;
      if (n < p.N) {
        __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(p.out) + (int64_t)blockIdx.y * p.stride_om;
        const float scale = (MODE == MODE_DOWNSUM) ? p.routed_scaling : 1.f;
        op[n] = __float2bfloat16(any_row ? v * scale : 0.f);
      }
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

template <int MODE, typename AT>
static int launch_gemv(const GemvParams& p, dim3 grid, cudaStream_t stream) {
  const int nw = pick_warps(p.K);
  const size_t smem = gemv_smem_bytes(p.K, nw);
  auto kern = gemv_kernel<MODE, AT>;
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
  p.stride_ww = g.stride_ww; p.stride_sg = g.stride_sg; p.stride_zg = g.stride_zg; p.I = 0;
  p.mul_routed_weight = g.mul_routed_weight; p.scale_bf16 = g.scale_bf16; p.routed_scaling = 1.f;
  p.err = g.err;
  dim3 grid((g.N + 127) / 128, g.R);
  return launch_gemv<MODE_PLAIN, __nv_bfloat16>(p, grid, g.stream);
}

int gemv_gateup_silu(const GemvArgs& g, int I, float* h, int64_t stride_hm) {
  if (g.R <= 0) return kOk;
  if (g.K <= 0 || g.K % kGroup != 0 || I <= 0 || I % 4 != 0) return kErrShape;
  if (g.stride_ww % 4 != 0 || g.stride_sg % 4 != 0 || g.stride_ww < 2 * I || g.stride_sg < 2 * I) return kErrAlign;
  GemvParams p{};
  p.a = g.a; p.stride_am = g.stride_am; p.map = g.map; p.ids = g.ids; p.topk_w = g.topk_w;
  p.out = h; p.stride_om = stride_hm; p.R = g.R; p.N = 2 * I; p.K = g.K; p.top_k = g.top_k;
  p.stride_ww = g.stride_ww; p.stride_sg = g.stride_sg; p.stride_zg = g.stride_zg; p.I = I;
  p.mul_routed_weight = 0; p.scale_bf16 = g.scale_bf16; p.routed_scaling = 1.f; p.err = g.err;
  dim3 grid((I + 63) / 64, g.R);
  return launch_gemv<MODE_GATEUP, __nv_bfloat16>(p, grid, g.stream);
}

int gemv_down_sum(const GemvArgs& g, int M, float routed_scaling) {
  if (M <= 0) return kOk;
  if (g.K <= 0 || g.K % kGroup != 0 || g.N <= 0 || g.N % 4 != 0) return kErrShape;
  if (g.stride_ww % 4 != 0 || g.stride_sg % 4 != 0 || g.stride_ww < g.N || g.stride_sg < g.N) return kErrAlign;
  GemvParams p{};
  p.a = g.a; p.stride_am = g.stride_am; p.map = g.map; p.ids = g.ids; p.topk_w = g.topk_w;
  p.out = g.out; p.stride_om = g.stride_om; p.R = M * g.top_k; p.N = g.N; p.K = g.K; p.top_k = g.top_k;
  p.stride_ww = g.stride_ww; p.stride_sg = g.stride_sg; p.stride_zg = g.stride_zg; p.I = 0;
  p.mul_routed_weight = 1; p.scale_bf16 = g.scale_bf16; p.routed_scaling = routed_scaling; p.err = g.err;
  dim3 grid((g.N + 127) / 128, M);
  return launch_gemv<MODE_DOWNSUM, float>(p, grid, g.stream);
}

}  // namespace w2a16
