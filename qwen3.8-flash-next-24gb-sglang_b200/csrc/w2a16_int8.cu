// INT8 dense projection GEMV (sm_100a, CUDA cores, dp2a on whole weight bytes).
//
// y[m, n] = sum_k (q[k, n] - zero) * s[k / group, n] * x[m, k]
// Weights int32 [K/4, N]: byte i of word kw = value 4*kw + i (auto_gptq INT8 packing,
// scripts/requant_int8.py:32-50). One 16-byte load per lane covers 4 columns x 4 k; dp2a.lo/hi
// multiply the four weight bytes by 16-bit fixed-point activations (power-of-two scale per 128
// values, as in the W2 kernels). The zero point folds as T - zero * sum x_fixed per 32-k quarter.
//
// Split-K over CTAs (256 k per CTA, 8 warps x 32 k); each CTA writes fp32 partials, the last CTA of
// a column block (atomic ticket) sums them in k-slice order -> deterministic bf16 output. The
// ticket counters are reset by that last CTA, so the workspace stays reusable without a memset.
#include "w2a16_kernels.h"

namespace w2a16 {

namespace {
constexpr int kTokPerCta = 4;
constexpr int kSlice = 256;     // k per CTA
constexpr int kWarps = 8;       // 32 k each

struct I8Params {
  const __nv_bfloat16* x; int64_t stride_xm;
  const int32_t* qw; const __half* scales; int group; int zero;
  int M, K, N;
  __nv_bfloat16* y; int64_t stride_ym;
  float* part;         // [nslices][M][N]
  unsigned* tickets;   // [N/128 * ceil(M/4)]
};
}  // namespace

__global__ void __launch_bounds__(256) int8_gemv_kernel(I8Params p) {
  __shared__ __align__(16) int16_t xq[kTokPerCta][kSlice];
  __shared__ int xsum_q[kTokPerCta][kWarps];
  __shared__ float xscale[kTokPerCta][2];
  __shared__ float red[kTokPerCta][kWarps][128];
  __shared__ int is_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cb = blockIdx.x, ks = blockIdx.y, mz = blockIdx.z;
  const int m0 = mz * kTokPerCta;
  const int mt = min(kTokPerCta, p.M - m0);
  const int k0 = ks * kSlice;
  const int nslices = gridDim.y;

  // activation prep: one warp per (token, 128-wide x-group)
  for (int t = warp; t < mt * 2; t += kWarps) {
    const int m = t >> 1, xg = t & 1;
    const int kb = k0 + xg * 128;
    if (kb >= p.K) continue;
    const __nv_bfloat16* src = p.x + (int64_t)(m0 + m) * p.stride_xm + kb;
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __bfloat162float(src[4 * lane + i]);
    float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    int E = 0;
    if (mx > 0.f) frexpf(mx, &E);
    const float inv = ldexpf(1.f, 15 - E);
    int s = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int q = __float2int_rn(v[i] * inv);
      q = max(-32767, min(32767, q));
      xq[m][xg * 128 + 4 * lane + i] = (int16_t)q;
      s += q;
    }
    // quarter sums: lanes 8c .. 8c+7 cover quarter c of this x-group
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((lane & 7) == 0) xsum_q[m][xg * 4 + (lane >> 3)] = s;
    if (lane == 0) xscale[m][xg] = ldexpf(1.f, E - 15);
  }
  __syncthreads();

  const int q = cb * 32 + lane;
  const int kq = k0 + 32 * warp;                     // first k of this warp's quarter
  const bool active = (4 * q < p.N) && (kq < p.K);
  float out[kTokPerCta][4];
#pragma unroll
  for (int m = 0; m < kTokPerCta; ++m)
#pragma unroll
    for (int c = 0; c < 4; ++c) out[m][c] = 0.f;
  if (active) {
    uint4 W[8];
    const int32_t* wp = p.qw + (int64_t)(kq >> 2) * p.N + 4 * q;
#pragma unroll
    for (int i = 0; i < 8; ++i) W[i] = __ldg(reinterpret_cast<const uint4*>(wp + (int64_t)i * p.N));
    float sc[4] = {1.f, 1.f, 1.f, 1.f};
    if (p.group < p.K) {
      const __half* sp = p.scales + (int64_t)(kq / p.group) * p.N + 4 * q;
#pragma unroll
      for (int c = 0; c < 4; ++c) sc[c] = __half2float(sp[c]);
    }
    const uint32_t* xp32 = reinterpret_cast<const uint32_t*>(&xq[0][0]);
    for (int m = 0; m < mt; ++m) {
      int acc[4] = {0, 0, 0, 0};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        // k = kq + 4i .. +3 -> x pairs (k, k+1), (k+2, k+3)
        const int kl = 32 * warp + 4 * i;
        const uint32_t xa = xp32[(m * kSlice + kl) >> 1];
        const uint32_t xb = xp32[(m * kSlice + kl + 2) >> 1];
        acc[0] = dp2a_hi(xb, W[i].x, dp2a_lo(xa, W[i].x, acc[0]));
        acc[1] = dp2a_hi(xb, W[i].y, dp2a_lo(xa, W[i].y, acc[1]));
        acc[2] = dp2a_hi(xb, W[i].z, dp2a_lo(xa, W[i].z, acc[2]));
        acc[3] = dp2a_hi(xb, W[i].w, dp2a_lo(xa, W[i].w, acc[3]));
      }
      const int zfold = -p.zero * xsum_q[m][warp];
      const float es = xscale[m][warp >> 2];
#pragma unroll
      for (int c = 0; c < 4; ++c) out[m][c] = (float)(acc[c] + zfold) * es * sc[c];
    }
  }
#pragma unroll
  for (int m = 0; m < kTokPerCta; ++m)
#pragma unroll
    for (int c = 0; c < 4; ++c) red[m][warp][lane * 4 + c] = out[m][c];
  __syncthreads();

  // CTA partial for this k-slice
  for (int t = threadIdx.x; t < mt * 128; t += blockDim.x) {
    const int m = t >> 7, col = t & 127;
    const int n = cb * 128 + col;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[m][w][col];
    if (n < p.N) p.part[((int64_t)ks * p.M + (m0 + m)) * p.N + n] = v;
  }
  // Ticket: the CTA barrier orders every thread's partial before thread 0's acquire-release add, which
  // publishes them and, in the CTA that takes the last ticket, orders the other slices' partials before
  // its reads (after the second barrier). No full fences: they stall for microseconds under load.
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* t = p.tickets + (int64_t)mz * gridDim.x + cb;
    unsigned prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;\n" : "=r"(prev) : "l"(t) : "memory");
    is_last = (prev == (unsigned)(nslices - 1));
  }
  __syncthreads();
  if (!is_last) return;
  for (int t = threadIdx.x; t < mt * 128; t += blockDim.x) {
    const int m = t >> 7, col = t & 127;
    const int n = cb * 128 + col;
    if (n >= p.N) continue;
    float v = 0.f;
    for (int s = 0; s < nslices; ++s) v += __ldcg(p.part + ((int64_t)s * p.M + (m0 + m)) * p.N + n);
    if (p.group >= p.K) v *= __half2float(p.scales[n]);
    p.y[(int64_t)(m0 + m) * p.stride_ym + n] = __float2bfloat16(v);
  }
  if (threadIdx.x == 0) p.tickets[(int64_t)mz * gridDim.x + cb] = 0u;
}

// Workspace: ticket counters [ceil(M/4)][N/128] (16-byte padded), then fp32 partials [slices][M][N].
static size_t tickets_bytes(int M, int N) {
  const size_t ncb = (size_t)(N + 127) / 128, nz = (size_t)(M + kTokPerCta - 1) / kTokPerCta;
  return (ncb * nz * 4 + 15) & ~size_t(15);
}

size_t int8_workspace_bytes(int M, int K, int N) {
  const size_t nslices = (size_t)(K + kSlice - 1) / kSlice;
  return tickets_bytes(M, N) + nslices * (size_t)M * (size_t)N * 4;
}

int int8_gemv(const Int8Args& a, void* workspace, size_t workspace_bytes) {
  if (a.M <= 0) return kOk;
  if (a.K <= 0 || a.K % 128 != 0 || a.N <= 0 || a.N % 4 != 0) return kErrShape;
  if (a.group <= 0 || a.group % 128 != 0 || a.K % a.group != 0) return kErrShape;
  if (!a.x || !a.qweight || !a.scales || !a.y) return kErrArg;
  if ((reinterpret_cast<uintptr_t>(a.qweight) & 15u)) return kErrAlign;
  if (!workspace || workspace_bytes < int8_workspace_bytes(a.M, a.K, a.N)) return kErrWorkspace;
  I8Params p{};
  p.x = static_cast<const __nv_bfloat16*>(a.x); p.stride_xm = a.stride_xm;
  p.qw = a.qweight; p.scales = static_cast<const __half*>(a.scales); p.group = a.group; p.zero = a.zero;
  p.M = a.M; p.K = a.K; p.N = a.N;
  p.y = static_cast<__nv_bfloat16*>(a.y); p.stride_ym = a.stride_ym;
  const int nslices = (a.K + kSlice - 1) / kSlice;
  const int ncb = (a.N + 127) / 128, nz = (a.M + kTokPerCta - 1) / kTokPerCta;
  char* ws = static_cast<char*>(workspace);
  if (reinterpret_cast<uintptr_t>(ws) & 15u) return kErrAlign;
  p.tickets = reinterpret_cast<unsigned*>(ws);
  p.part = reinterpret_cast<float*>(ws + tickets_bytes(a.M, a.N));
  int8_gemv_kernel<<<dim3(ncb, nslices, nz), 256, 0, a.stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace w2a16
