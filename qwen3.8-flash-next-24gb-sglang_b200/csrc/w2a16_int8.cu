// INT8 dense projection GEMV (sm_100a, CUDA cores, dp2a on whole weight bytes).
//
// y[m, n] = sum_k (q[k, n] - zero) * s[k / group, n] * x[m, k]
// Weights int32 [K/4, N]: byte i of word kw = value 4*kw + i (auto_gptq INT8 packing,
// scripts/requant_int8.py:32-50). One 16-byte load per lane covers 4 columns x 4 k; dp2a.lo/hi
// multiply the four weight bytes by 16-bit fixed-point activations (power-of-two scale per 128
// values, as in the W2 kernels). The zero point folds as T - zero * sum x_fixed per 32-k quarter.
//
// Split-K inside a thread-block cluster: the S <= 8 CTAs of a cluster take the K slices of one block of
// 128 columns (8 warps x slice/8 k each); every CTA leaves its 128-column partial in shared memory and,
// after a cluster barrier, cluster rank 0 adds the S partials in rank order through distributed shared
// memory -> deterministic bf16 output, no workspace, no atomics. Launched with programmatic stream
// serialisation: the weight loads are issued before the kernel waits for the previous one, so the
// 16-byte-per-lane weight stream overlaps that kernel's tail (the weights are never written by a kernel
// that triggers this one early).
#include <cooperative_groups.h>

#include "w2a16_kernels.h"

namespace w2a16 {

namespace {
namespace cg = cooperative_groups;
constexpr int kTokPerCta = 4;
constexpr int kWarps = 8;
constexpr int kMaxCluster = 8;
constexpr int kMaxSlice = 2048;   // k per CTA (K <= 16384 in 8-CTA clusters)
constexpr int kBatches = 2;       // 32-k batches of weights a warp holds in registers at a time

struct I8Params {
  const __nv_bfloat16* x; int64_t stride_xm;
  const int32_t* qw; const __half* scales; int group; int zero;
  int M, K, N, slice;
  __nv_bfloat16* y; int64_t stride_ym;
  // expert parallelism: x = the sum of the ranks' tagged rows of the exchange channel's call *xepoch (rows of
  // K values) in this rank's buffer, each word used once it holds that call
  const uint64_t* xpeers; size_t xtag_off; unsigned* xepoch;
  int xrank, xworld, xn_max; unsigned xspin; unsigned* err;
};
}  // namespace

// kPeers: x from the exchange channel; the plain variant carries none of it.
template <bool kPeers>
__global__ void __launch_bounds__(256) int8_gemv_kernel(I8Params p) {
  __shared__ __align__(16) int16_t xq[kTokPerCta][kMaxSlice];
  __shared__ int xsum_q[kTokPerCta][kMaxSlice / 32];
  __shared__ float xscale[kTokPerCta][kMaxSlice / 128];
  __shared__ float red[kTokPerCta][kWarps][128];
  __shared__ float cpart[kTokPerCta][128];
  cg::cluster_group cluster = cg::this_cluster();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cb = blockIdx.x, ks = blockIdx.y, mz = blockIdx.z;
  const int m0 = mz * kTokPerCta;
  const int mt = min(kTokPerCta, p.M - m0);
  const int k0 = ks * p.slice;
  const int wk = p.slice / kWarps;                   // k of this warp: a multiple of 32
  const int nb = wk / 32;
  const int q = cb * 32 + lane;                      // column quad

  // this warp's weights kBatches x 32 k at a time; the first ones (static data) before the dependency wait
  uint4 W[kBatches][8];
  float sc[kBatches][4];
  auto load = [&](int sb) {
#pragma unroll
    for (int b = 0; b < kBatches; ++b) {
      const int bb = sb * kBatches + b;
      const int kq = k0 + warp * wk + 32 * bb;
      sc[b][0] = sc[b][1] = sc[b][2] = sc[b][3] = 1.f;
      if (bb < nb && 4 * q < p.N && kq < p.K) {
        const int32_t* wp = p.qw + (int64_t)(kq >> 2) * p.N + 4 * q;
#pragma unroll
        for (int i = 0; i < 8; ++i) W[b][i] = __ldg(reinterpret_cast<const uint4*>(wp + (int64_t)i * p.N));
        if (p.group < p.K) {
          const __half* sp = p.scales + (int64_t)(kq / p.group) * p.N + 4 * q;
#pragma unroll
          for (int c = 0; c < 4; ++c) sc[b][c] = __half2float(sp[c]);
        }
      }
    }
  };
  load(0);
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  const unsigned long long* xsum = nullptr;
  unsigned e_in = 0, budget = p.xspin;
  if (kPeers) {
    e_in = ld_relaxed_gpu_u32(p.xepoch);
    xsum = reinterpret_cast<const unsigned long long*>(p.xpeers[p.xrank] + p.xtag_off) +
           (size_t)(e_in & 1u) * p.xworld * (p.xn_max / 2);
  }

  // activation prep: one warp per (token, 128-wide x-group) of the slice
  const int ng = p.slice / 128;
  for (int t = warp; t < mt * ng; t += kWarps) {
    const int m = t / ng, xg = t - m * ng;
    const int kb = k0 + xg * 128;
    if (kb >= p.K) continue;
    float v[4];
    if (!kPeers) {
      const __nv_bfloat16* src = p.x + (int64_t)(m0 + m) * p.stride_xm + kb;
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __bfloat162float(src[4 * lane + i]);
    } else {
      // the ranks' rows in rank order, summed in fp32 and rounded to bf16 as the all-reduce does
      const size_t w0 = ((size_t)(m0 + m) * p.K + kb + 4 * lane) / 2;
      float s[4] = {0.f, 0.f, 0.f, 0.f};
      for (int r = 0; r < p.xworld; ++r) {
        const unsigned long long* row = xsum + (size_t)r * (p.xn_max / 2) + w0;
        const float2 a0 = bf16x2_to_float2(wait_tagged(row, e_in, budget, p.err));
        const float2 a1 = bf16x2_to_float2(wait_tagged(row + 1, e_in, budget, p.err));
        s[0] += a0.x; s[1] += a0.y; s[2] += a1.x; s[3] += a1.y;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __bfloat162float(__float2bfloat16(s[i]));
    }
    float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    mx = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(mx)));
    const int E = (mx > 0.f ? frexp_exponent(mx) : 0) - 15;
    const float inv = pow2f(-E);
    int s = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int qv = __float2int_rn(v[i] * inv);
      qv = max(-32767, min(32767, qv));
      xq[m][xg * 128 + 4 * lane + i] = (int16_t)qv;
      s += qv;
    }
    // quarter sums: lanes 8c .. 8c+7 cover quarter c of this x-group
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((lane & 7) == 0) xsum_q[m][xg * 4 + (lane >> 3)] = s;
    if (lane == 0) xscale[m][xg] = pow2f(E);
  }
  __syncthreads();

  float out[kTokPerCta][4];
#pragma unroll
  for (int m = 0; m < kTokPerCta; ++m)
#pragma unroll
    for (int c = 0; c < 4; ++c) out[m][c] = 0.f;
  const uint32_t* xp32 = reinterpret_cast<const uint32_t*>(&xq[0][0]);
  const int nsb = (nb + kBatches - 1) / kBatches;
  for (int sb = 0; sb < nsb; ++sb) {
   if (sb > 0) load(sb);
#pragma unroll
   for (int b = 0; b < kBatches; ++b) {
    const int kl0 = warp * wk + 32 * (sb * kBatches + b);   // k within the slice
    if (sb * kBatches + b < nb && 4 * q < p.N && k0 + kl0 < p.K) {
      for (int m = 0; m < mt; ++m) {
        int acc[4] = {0, 0, 0, 0};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          // k = kl0 + 4i .. +3 -> x pairs (k, k+1), (k+2, k+3)
          const int kl = kl0 + 4 * i;
          const uint32_t xa = xp32[(m * kMaxSlice + kl) >> 1];
          const uint32_t xb = xp32[(m * kMaxSlice + kl + 2) >> 1];
          acc[0] = dp2a_hi(xb, W[b][i].x, dp2a_lo(xa, W[b][i].x, acc[0]));
          acc[1] = dp2a_hi(xb, W[b][i].y, dp2a_lo(xa, W[b][i].y, acc[1]));
          acc[2] = dp2a_hi(xb, W[b][i].z, dp2a_lo(xa, W[b][i].z, acc[2]));
          acc[3] = dp2a_hi(xb, W[b][i].w, dp2a_lo(xa, W[b][i].w, acc[3]));
        }
        const int zfold = -p.zero * xsum_q[m][kl0 >> 5];
        const float es = xscale[m][kl0 >> 7];
#pragma unroll
        for (int c = 0; c < 4; ++c) out[m][c] += (float)(acc[c] + zfold) * es * sc[b][c];
      }
    }
   }
  }
#pragma unroll
  for (int m = 0; m < kTokPerCta; ++m)
#pragma unroll
    for (int c = 0; c < 4; ++c) red[m][warp][lane * 4 + c] = out[m][c];
  __syncthreads();
  // this CTA's partial for its k-slice, warps in order
  for (int t = threadIdx.x; t < mt * 128; t += blockDim.x) {
    const int m = t >> 7, col = t & 127;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[m][w][col];
    cpart[m][col] = v;
  }
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  cluster.sync();
  if (cluster.block_rank() == 0) {
    const int S = (int)cluster.num_blocks();
    for (int t = threadIdx.x; t < mt * 128; t += blockDim.x) {
      const int m = t >> 7, col = t & 127;
      const int n = cb * 128 + col;
      if (n >= p.N) continue;
      float v = 0.f;
      for (int r = 0; r < S; ++r) v += cluster.map_shared_rank(&cpart[0][0], r)[t];
      if (p.group >= p.K) v *= __half2float(p.scales[n]);
      p.y[(int64_t)(m0 + m) * p.stride_ym + n] = __float2bfloat16(v);
    }
  }
  cluster.sync();                                    // every partial stays readable until rank 0 is done
}

// No workspace is needed any more; the entry point keeps its workspace arguments.
size_t int8_workspace_bytes(int M, int K, int N) {
  (void)M; (void)K; (void)N;
  return 256;
}

namespace {
int launch_int8(const Int8Args& a, const PeerExchange* xin, unsigned* err) {
  if (a.M <= 0) return kOk;
  if (a.K <= 0 || a.K % 128 != 0 || a.N <= 0 || a.N % 4 != 0) return kErrShape;
  if (a.group <= 0 || a.group % 128 != 0 || a.K % a.group != 0) return kErrShape;
  if ((!a.x && !xin) || !a.qweight || !a.scales || !a.y) return kErrArg;
  if (xin && (!xin->peers || !xin->epoch || xin->world <= 0 || xin->rank < 0 || xin->rank >= xin->world ||
              xin->n_max % 8 || (size_t)a.M * a.K > (size_t)xin->n_max || xin->tag_off % 16))
    return kErrArg;
  if ((reinterpret_cast<uintptr_t>(a.qweight) & 15u)) return kErrAlign;
  // S slices of a multiple of 256 k each (at most kMaxSlice), one cluster of S CTAs per column block
  int S = (a.K + 255) / 256;
  if (S > kMaxCluster) S = kMaxCluster;
  const int slice = ((a.K + S - 1) / S + 255) / 256 * 256;
  if (slice > kMaxSlice) return kErrShape;
  S = (a.K + slice - 1) / slice;
  I8Params p{};
  p.x = static_cast<const __nv_bfloat16*>(a.x); p.stride_xm = a.stride_xm;
  p.qw = a.qweight; p.scales = static_cast<const __half*>(a.scales); p.group = a.group; p.zero = a.zero;
  p.M = a.M; p.K = a.K; p.N = a.N; p.slice = slice;
  p.y = static_cast<__nv_bfloat16*>(a.y); p.stride_ym = a.stride_ym;
  if (xin) {
    p.xpeers = xin->peers;
    p.xtag_off = xin->tag_off;
    p.xrank = xin->rank;
    p.xepoch = xin->epoch;
    p.xworld = xin->world;
    p.xn_max = xin->n_max;
    p.xspin = xin->spin_limit ? xin->spin_limit : kPeerSpinLimit;
    p.err = err;
  }
  const int ncb = (a.N + 127) / 128, nz = (a.M + kTokPerCta - 1) / kTokPerCta;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(ncb, S, nz);
  cfg.blockDim = dim3(256);
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = S;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, xin ? int8_gemv_kernel<true> : int8_gemv_kernel<false>, p) == cudaSuccess
             ? kOk : kErrLaunch;
}
}  // namespace

int int8_gemv(const Int8Args& a, void* workspace, size_t workspace_bytes) {
  (void)workspace; (void)workspace_bytes;
  return launch_int8(a, nullptr, nullptr);
}

int int8_gemv_from_peers(const Int8Args& a, const PeerExchange& xin, unsigned* err) {
  return launch_int8(a, &xin, err);
}

}  // namespace w2a16
