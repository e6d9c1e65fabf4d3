// Batched decode MoE layer (M >= 16 tokens) on the 5th-generation tensor cores (sm_100a tcgen05): the routed
// rows are grouped by expert, so each resident expert's weights cross HBM once per call however many of the
// tokens route to it (the per-token fused layer streams an expert once per routed row). Same computation as
// the composite of patches/ncontig_gemv.py:218-238: gate_up GEMV, SiLU*mul, down GEMV * routed weight,
// top-k sum, with the slot-table indirection of row_arena.py.
//
// route_kernel (one CTA): the live routed rows (slot >= 0) sorted by (slot, row) and cut into groups of at
// most kGN rows of one expert.
//
// proj_kernel<kGateUp> (persistent, one CTA per SM): work items (group, tile of 128 weight columns -- gate_up:
// 64 gate columns and the matching 64 up columns; down: 128 output columns), dealt round-robin. A producer warp
// streams each item's codes, scales and zero points through a ring of shared-memory stages with tensor copies
// (the fused layer's arena maps). Per 128-value quantization group along K:
//   * warps 8-15 expand the codes to bf16(128 + q) -- exact -- straight into tensor memory as the MMA's A
//     operand (the tile's column r is TMEM lane r; one 16-value word is 8 columns, one tcgen05.st);
//   * warps 4-7 stage the group's rows of the activation (x for gate_up, h for down) in shared memory as the
//     B operand, with the rows' sums and the tile's scales and zero points;
//   * two MMA warps, taking alternate groups, issue 8 tcgen05.mma (A from tensor memory, M = 128 columns,
//     N = 16 rows, K = 16, fp32 accumulation in tensor memory) and commit them to an mbarrier;
//   * warps 0-3 read the accumulators (tcgen05.ld) and fold them into registers:
//     acc += s * (D - (128 + zp) * sum x), the reference's zero-point fold (gemv/moe_gemv_int2_tab.py:61-66)
//     applied per group with its scale.
// Four operand and accumulator buffers rotate between groups, handed over with mbarriers (operands ready,
// MMA done, accumulator read), so every role works on a different group at a time. Within each 16-value word
// the MMA's K order is permuted (position 2j = value j, 2j + 1 = value j + 8, which is what one LOP3 per pair
// yields); the B operand is staged in the same order. At decode sizes an expert has only a few rows per call,
// so N = 16 MMAs leave the tensor pipe mostly idle (about 5 % active); the path pays where the per-token
// path re-reads each expert many times, from about 64 tokens.
// Epilogues: gate_up -> h = silu(gate) * up in bf16 per routed row; down -> routed weight * y row in fp32.
//
// sum_kernel: y[m] = routed_scaling * (sum of the token's live y rows in routing order), deterministic.
#include <climits>
#include <cuda.h>
#include <cudaTypedefs.h>

#include "w2a16_kernels.h"

namespace w2a16 {
namespace {

constexpr int kGN = 16;                          // MMA N: rows of one group
constexpr int kTileCols = 128;                   // MMA M: weight columns of a tile
constexpr int kCompute = 512;                    // warps 0-3 fold, 4-7 stage B and the scales, 8-15 expand codes
constexpr int kWriters = kCompute - 128;          // threads that write a group's operands (warps 4-15)
constexpr int kMmaWarps = 2;                     // MMA issuers, taking alternate groups
constexpr int kGThreads = kCompute + 32 + 32 * kMmaWarps;   // + the producer warp and the MMA warps
constexpr int kAcols = kGroup / 2;               // TMEM columns of one group of the A operand (bf16 pairs)
constexpr int kWordRows = kGroup / 16;           // 16-value word rows of a group
constexpr int kBBytes = kGN * kGroup * 2;        // one group of the B operand (bf16)
constexpr int kGURing = 16, kDNRing = 8;
// Ring stages (offsets multiples of 128 bytes, as tensor copies require):
//   gate_up, 2 groups x (64 gate + 64 up columns): codes 2 x 4 KB [copy][word row][half][32 columns],
//     scales 2 x 256 B at 8192 [copy][group][half][32], zero windows 64 B at 8704 [group][half][16 bytes];
//   down, 4 groups x 128 columns: codes 4 x 4 KB [copy][word row][32 columns], scales 4 x 256 B at 16384
//     [copy][group][32], zero windows 2 x 64 B at 17408 (stride 128) [window][group][16 bytes].
constexpr int kGUStage = 8832, kGUScale = 8192, kGUZero = 8704;
constexpr int kDNStage = 17664, kDNScale = 16384, kDNZero = 17408;
constexpr int kMaxGroupedRows = 1024;            // routed rows per launch
constexpr int kGroupedChunk = 128;               // tokens per launch
constexpr unsigned kGWait = 1u << 17;            // suspending mbarrier tries before a wait gives up
constexpr int kNB = 4;                           // operand / accumulator buffers in flight
constexpr int kTmemCols = 512;                   // A: kNB buffers of kAcols columns; then kNB accumulators of kGN
// kind::f16 instruction descriptor: fp32 accumulator, bf16 A and B, both K-major, N = 16, M = 128
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kGN >> 3) << 17) |
                            ((uint32_t)(kTileCols >> 4) << 24);

__host__ __device__ constexpr int ring_bytes(bool gu) { return gu ? kGURing * kGUStage : kDNRing * kDNStage; }
// mbarriers (full, empty per stage; ready, mma, tfree per buffer), tensor-memory address, row sums [kNB][kGN],
// scales and zero points [kNB][128], gate_up's up-half exchange [64][kGN]
__host__ __device__ constexpr int small_bytes(bool gu) {
  return (2 * (gu ? kGURing : kDNRing) + 3 * kNB) * 8 + 16 + kNB * kGN * 4 + kNB * kTileCols * 8 + 64 * kGN * 4;
}
__host__ __device__ constexpr int proj_smem(bool gu) { return kNB * kBBytes + ring_bytes(gu) + small_bytes(gu); }

// Route tables in the workspace: [0] groups, then gslot, gstart, gcnt, order (R entries each) from int 16.
struct RouteView {
  int* base;
  int R;
  __host__ __device__ int* gslot() const { return base + 16; }
  __host__ __device__ int* gstart() const { return base + 16 + R; }
  __host__ __device__ int* gcnt() const { return base + 16 + 2 * R; }
  __host__ __device__ int* order() const { return base + 16 + 3 * R; }
};

struct ProjParams {
  CUtensorMap tm[3];          // codes, scales, zero windows of this projection (arena maps)
  int* route;                 // route tables (RouteView layout)
  int R;
  const __nv_bfloat16* act;   // gate_up: x [M, H]; down: h [R, I]
  int64_t act_stride;         // elements per activation row
  int act_row_div;            // routed row r reads activation row r / act_row_div
  int K, N;                   // reduction length (H or I), weight columns (2I or H)
  int I;                      // h columns (gate_up output)
  int has_zeros, scale_bf16;
  const float* topk_w;        // down: routed weights [R]
  __nv_bfloat16* hout;        // gate_up: h [R, I]
  float* yrows;               // down: [R, H]
  unsigned* err;
};

__device__ __forceinline__ uint32_t s_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void g_mbar_init(uint32_t bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void g_mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void g_mbar_arrive_tx(uint32_t bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
// Bounded wait for the phase of the given parity (error bit 1 when it gives up).
__device__ __forceinline__ void g_mbar_wait(uint32_t bar, unsigned parity, unsigned* err) {
  for (unsigned it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return;
    if (it > kGWait) {
      flag_error(err, 2u);
      return;
    }
  }
}
__device__ __forceinline__ void g_tma_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void g_tma_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void fold_sync() { asm volatile("bar.sync 2, 128;\n" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, no swizzle: core matrices of 8 rows x 16 bytes, the two 16-byte
// halves of a K = 16 slice 128 bytes apart (leading byte offset), 8-row groups 256 bytes apart (stride byte
// offset); descriptor version 1.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) |
         (1ull << 46);
}
// byte offset of (row, K half) of a K = 16 slice in that layout
__device__ __forceinline__ int canon_off(int row, int half) { return (row >> 3) * 256 + half * 128 + (row & 7) * 16; }

// ----------------------------------------------------------------------------------------------- routing
__global__ void __launch_bounds__(1024) route_kernel(const int32_t* ids, const int32_t* slots, int E, int S, int R,
                                                     int* route, unsigned* err) {
  __shared__ int key[kMaxGroupedRows];
  __shared__ int srt[kMaxGroupedRows];
  __shared__ int start[kMaxGroupedRows];
  const RouteView rv{route, R};
  const int t = threadIdx.x;
  for (int r = t; r < R; r += blockDim.x) {
    const int e = ids[r];
    int sl = -1;
    if (e < 0 || e >= E) {
      flag_error(err, 1u);
    } else {
      sl = slots[e];
      if (sl >= S) {                                   // past the arena: masked, flagged
        flag_error(err, 1u);
        sl = -1;
      }
    }
    key[r] = sl >= 0 ? sl : INT_MAX;
  }
  __syncthreads();
  for (int r = t; r < R; r += blockDim.x) {           // rank by (slot, row): live rows first
    const int k = key[r];
    int rank = 0;
    for (int j = 0; j < R; ++j) {
      const int kj = key[j];
      rank += (kj < k) || (kj == k && j < r);
    }
    srt[rank] = r;
  }
  __syncthreads();
  for (int q = t; q < R; q += blockDim.x) {           // a group starts every kGN rows of one slot
    const int k = key[srt[q]];
    int st = 0;
    if (k != INT_MAX) {
      int first = q;
      while (first > 0 && key[srt[first - 1]] == k) --first;
      st = (q - first) % kGN == 0;
    }
    start[q] = st;
  }
  __syncthreads();
  for (int q = t; q < R; q += blockDim.x) {
    rv.order()[q] = srt[q];
    if (!start[q]) continue;
    int gid = 0;
    for (int j = 0; j < q; ++j) gid += start[j];
    const int k = key[srt[q]];
    int cnt = 1;
    while (q + cnt < R && cnt < kGN && !start[q + cnt] && key[srt[q + cnt]] == k) ++cnt;
    rv.gslot()[gid] = k;
    rv.gstart()[gid] = q;
    rv.gcnt()[gid] = cnt;
  }
  if (t == 0) {
    int n = 0;
    for (int j = 0; j < R; ++j) n += start[j];
    route[0] = n;
  }
}

// ----------------------------------------------------------------------------------------------- projection
template <bool kGU>
__global__ void __launch_bounds__(kGThreads, 1) proj_kernel(const __grid_constant__ ProjParams p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  constexpr int kNS = kGU ? kGURing : kDNRing;
  constexpr int kStage = kGU ? kGUStage : kDNStage;
  constexpr int kGPS = kGU ? 2 : 4;                   // groups per stage
  unsigned char* bbuf = smem;                         // B operand, kNB buffers
  unsigned char* ring = smem + kNB * kBBytes;
  unsigned char* small = ring + ring_bytes(kGU);
  const uint32_t bars = s_u32(small);                 // full[kNS], empty[kNS], ready[kNB], mma[kNB], tfree[kNB]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(small + (2 * kNS + 3 * kNB) * 8);
  float* bsum = reinterpret_cast<float*>(small + (2 * kNS + 3 * kNB) * 8 + 16);   // [kNB][kGN]
  float* sc = bsum + kNB * kGN;                        // [kNB][128]
  int* zc = reinterpret_cast<int*>(sc + kNB * kTileCols);   // [kNB][128]
  float* upx = reinterpret_cast<float*>(zc + kNB * kTileCols);   // [64][kGN]
  auto full = [&](int s) { return bars + 8u * s; };
  auto empty = [&](int s) { return bars + 8u * (kNS + s); };
  auto ready = [&](int b) { return bars + 8u * (2 * kNS + b); };
  auto mmab = [&](int b) { return bars + 8u * (2 * kNS + kNB + b); };
  auto tfree = [&](int b) { return bars + 8u * (2 * kNS + 2 * kNB + b); };
  // group gc uses buffer gc % kNB for the (gc / kNB)-th time: the phase parity of its barriers
  auto buf = [](unsigned gc) { return (int)(gc % kNB); };
  auto par = [](unsigned gc) { return (gc / kNB) & 1u; };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const RouteView rv{p.route, p.R};
  const int G = p.K / kGroup;
  const int nsteps = (G + kGPS - 1) / kGPS;
  const int ntiles = kGU ? p.I / 64 : p.N / kTileCols;
  const bool aligned = (s_u32(smem) & 1023u) == 0;
  constexpr int kProducerWarp = kCompute / 32, kMmaWarp = kProducerWarp + 1;

  if (warp == kProducerWarp && lane == 0) {
    for (int s = 0; s < kNS; ++s) {
      g_mbar_init(full(s), 1);
      g_mbar_init(empty(s), kWriters);
    }
    for (int b = 0; b < kNB; ++b) {
      g_mbar_init(ready(b), kWriters);
      g_mbar_init(mmab(b), 1);
      g_mbar_init(tfree(b), 128);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    for (int k = 0; k < 3; ++k)
      if (k < 2 || p.has_zeros) asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&p.tm[k])) : "memory");
    if (!aligned) flag_error(p.err, 4u);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(s_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = *tmem_slot;
  const int ngroups = p.route[0];
  const int nitems = ngroups * ntiles;

  if (warp == kProducerWarp) {
    // producer: the stages of this CTA's items, in order, by one lane
    if (lane == 0) {
      const bool hz = p.has_zeros != 0;
      const unsigned bytes = kGU ? (2 * 4096 + 2 * 256 + (hz ? 64 : 0)) : (4 * 4096 + 4 * 256 + (hz ? 128 : 0));
      int i = 0;
      for (int w = blockIdx.x; w < nitems; w += gridDim.x) {
        const int gi = w / ntiles, t = w - gi * ntiles;
        const int slot = rv.gslot()[gi];
        for (int s = 0; s < nsteps; ++s, ++i) {
          const int st = i % kNS, round = i / kNS;
          if (round > 0) g_mbar_wait(empty(st), (unsigned)(round - 1) & 1u, p.err);
          const uint32_t dst = s_u32(ring + (size_t)st * kStage);
          if (!aligned) {
            g_mbar_arrive(full(st));
            continue;
          }
          g_mbar_arrive_tx(full(st), bytes);
          if constexpr (kGU) {
            for (int c = 0; c < 2; ++c) {
              g_tma_4d(dst + c * 4096, &p.tm[0], 64 * t + 32 * c, 0, 16 * s, slot, full(st));
              g_tma_4d(dst + kGUScale + c * 256, &p.tm[1], 64 * t + 32 * c, 0, 2 * s, slot, full(st));
            }
            if (hz) g_tma_4d(dst + kGUZero, &p.tm[2], 16 * t, 0, 2 * s, slot, full(st));
          } else {
            for (int c = 0; c < 4; ++c) {
              g_tma_3d(dst + c * 4096, &p.tm[0], 128 * t + 32 * c, 32 * s, slot, full(st));
              g_tma_3d(dst + kDNScale + c * 256, &p.tm[1], 128 * t + 32 * c, 4 * s, slot, full(st));
            }
            if (hz)
              for (int z = 0; z < 2; ++z) g_tma_3d(dst + kDNZero + z * 128, &p.tm[2], 32 * t + 16 * z, 4 * s, slot, full(st));
          }
        }
      }
      // every copy has landed before the producer leaves
      for (int st = 0; st < kNS && st < i; ++st) {
        const int last = st + ((i - 1 - st) / kNS) * kNS;
        g_mbar_wait(full(st), (unsigned)(last / kNS) & 1u, p.err);
      }
    }
    return;
  }

  if (warp >= kMmaWarp) {
    // MMA issuers (one thread per warp takes every kMmaWarps-th group: one thread issues an MMA only every
    // few tens of cycles): per group, once its operands are in place and its accumulator buffer has been read
    if (lane == 0) {
      const unsigned q = (unsigned)(warp - kMmaWarp);
      unsigned gc = 0;
      for (int w = blockIdx.x; w < nitems; w += gridDim.x)
        for (int g = 0; g < G; ++g, ++gc) {
          if (gc % kMmaWarps != q) continue;
          const int b = buf(gc);
          g_mbar_wait(ready(b), par(gc), p.err);
          if (gc >= kNB) g_mbar_wait(tfree(b), par(gc - kNB), p.err);
          tc_after();
          const uint32_t b0 = s_u32(bbuf + b * kBBytes);
          const uint32_t dt = tmem + (uint32_t)(kNB * kAcols + b * kGN);
#pragma unroll
          for (int k16 = 0; k16 < kGroup / 16; ++k16) {
            const uint32_t at = tmem + (uint32_t)(b * kAcols + k16 * 8);
            const uint64_t bd = kmajor_desc(b0 + k16 * 512);
            asm volatile(
                "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(dt),
                "r"(at), "l"(bd), "r"(kIdesc), "r"(k16)
                : "memory");
          }
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(mmab(b))
                       : "memory");
        }
    }
    __syncwarp();
  } else if (warp < 4) {
    // ---------------------------------------------------------------- fold warps: thread r = tile column r
    unsigned gc = 0;
    float acc[kGN];
    for (int w = blockIdx.x; w < nitems; w += gridDim.x) {
      const int gi = w / ntiles, t = w - gi * ntiles;
      const int g0 = rv.gstart()[gi], cnt = rv.gcnt()[gi];
#pragma unroll
      for (int n = 0; n < kGN; ++n) acc[n] = 0.f;
      for (int g = 0; g < G; ++g, ++gc) {
        const int bx = buf(gc);
        g_mbar_wait(ready(bx), par(gc), p.err);         // this group's scales, zero points, row sums
        g_mbar_wait(mmab(bx), par(gc), p.err);          // and its accumulators
        tc_after();
        uint32_t d[kGN];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
            "%15}, [%16];\n"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]), "=r"(d[7]),
              "=r"(d[8]), "=r"(d[9]), "=r"(d[10]), "=r"(d[11]), "=r"(d[12]), "=r"(d[13]), "=r"(d[14]), "=r"(d[15])
            : "r"(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(kNB * kAcols + bx * kGN)));
        asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
        const float s = sc[bx * kTileCols + tid];
        const float zz = 128.f + (float)zc[bx * kTileCols + tid];
#pragma unroll
        for (int n = 0; n < kGN; ++n) acc[n] += s * (__uint_as_float(d[n]) - zz * bsum[bx * kGN + n]);
        tc_before();
        g_mbar_arrive(tfree(bx));                       // accumulators and row data of buffer bx are read
      }
      if constexpr (kGU) {
        // rows 0-63 gate, 64-127 up of the tile's 64 h-columns: h = silu(gate) * up
        if (tid >= 64)
#pragma unroll
          for (int n = 0; n < kGN; ++n) upx[(tid - 64) * kGN + n] = acc[n];
        fold_sync();
        if (tid < 64)
#pragma unroll
          for (int n = 0; n < kGN; ++n)
            if (n < cnt) {
              const int row = rv.order()[g0 + n];
              p.hout[(int64_t)row * p.I + 64 * t + tid] = __float2bfloat16(silu(acc[n]) * upx[tid * kGN + n]);
            }
        fold_sync();
      } else {
#pragma unroll
        for (int n = 0; n < kGN; ++n)
          if (n < cnt) {
            const int row = rv.order()[g0 + n];
            p.yrows[(int64_t)row * p.N + kTileCols * t + tid] = p.topk_w[row] * acc[n];
          }
      }
    }
  } else if (warp < 8) {
    // ---------------------------------------------------------------- staging warps: B, row sums, scales
    const bool sbf = p.scale_bf16 != 0, hz = p.has_zeros != 0;
    const int r = tid - 128;                            // tile column whose scale / zero point this thread takes
    const int bn = r >> 3, bs = r & 7;                  // B row r / 8, K = 16 slice r % 8 of every group
    int i = 0;
    unsigned gc = 0;
    for (int w = blockIdx.x; w < nitems; w += gridDim.x) {
      const int gi = w / ntiles;
      const int g0 = rv.gstart()[gi], cnt = rv.gcnt()[gi];
      const __nv_bfloat16* brow = nullptr;
      if (bn < cnt) brow = p.act + (int64_t)(rv.order()[g0 + bn] / p.act_row_div) * p.act_stride + bs * 16;
      uint4 pa = make_uint4(0, 0, 0, 0), pb = pa;
      if (brow) {
        pa = *reinterpret_cast<const uint4*>(brow);
        pb = *reinterpret_cast<const uint4*>(brow + 8);
      }
      for (int g = 0; g < G; ++g, ++gc) {
        const int s = g / kGPS, gs = g - s * kGPS;
        const int st = (i + s) % kNS;
        const int b = buf(gc);
        if (gc >= kNB) g_mbar_wait(tfree(b), par(gc - kNB), p.err);   // group gc - kNB folded (its MMA done)
        if (gs == 0) g_mbar_wait(full(st), (unsigned)((i + s) / kNS) & 1u, p.err);
        const unsigned char* stg = ring + (size_t)st * kStage;
        uint32_t raw;
        int zp = 2;
        if constexpr (kGU) {
          const int c = (r & 63) >> 5, half = r >> 6;
          raw = *reinterpret_cast<const uint16_t*>(stg + kGUScale + c * 256 + ((gs * 2 + half) * 32 + (r & 31)) * 2);
          if (hz) zp = (stg[kGUZero + (gs * 2 + half) * 16 + ((r & 63) >> 2)] >> (2 * (r & 3))) & 3;
        } else {
          raw = *reinterpret_cast<const uint16_t*>(stg + kDNScale + (r >> 5) * 256 + (gs * 32 + (r & 31)) * 2);
          if (hz) zp = (stg[kDNZero + (r >> 6) * 128 + gs * 16 + ((r & 63) >> 2)] >> (2 * (r & 3))) & 3;
        }
        sc[b * kTileCols + r] = sbf ? __bfloat162float(__ushort_as_bfloat16((unsigned short)raw))
                                    : __half2float(__ushort_as_half((unsigned short)raw));
        zc[b * kTileCols + r] = zp;
        // B: the prefetched slice in the permuted K order, and the row's sum over the group
        unsigned char* B = bbuf + b * kBBytes + bs * 512 + canon_off(bn, 0);
        *reinterpret_cast<uint4*>(B) = make_uint4(__byte_perm(pa.x, pb.x, 0x5410), __byte_perm(pa.x, pb.x, 0x7632),
                                                  __byte_perm(pa.y, pb.y, 0x5410), __byte_perm(pa.y, pb.y, 0x7632));
        *reinterpret_cast<uint4*>(B + 128) = make_uint4(__byte_perm(pa.z, pb.z, 0x5410), __byte_perm(pa.z, pb.z, 0x7632),
                                                        __byte_perm(pa.w, pb.w, 0x5410), __byte_perm(pa.w, pb.w, 0x7632));
        float sum = 0.f;
        const uint32_t v[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) sum += __uint_as_float(v[k] << 16) + __uint_as_float(v[k] & 0xFFFF0000u);
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        if (bs == 0) bsum[b * kGN + bn] = sum;
        if (brow && g + 1 < G) {                        // next group's slice
          pa = *reinterpret_cast<const uint4*>(brow + (g + 1) * kGroup);
          pb = *reinterpret_cast<const uint4*>(brow + (g + 1) * kGroup + 8);
        }
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");   // generic writes -> the MMA's reads
        g_mbar_arrive(ready(b));
        if (gs == kGPS - 1 || g == G - 1) g_mbar_arrive(empty(st));     // this thread is done with the stage
      }
      i += nsteps;
    }
  } else {
    // ---------------------------------------------------------------- expansion warps: codes -> A in TMEM
    // warp 8 + q takes TMEM lanes (tile columns) 32 (q % 4) .. + 31 and word rows q / 4, q / 4 + 2, ...
    const int r = 32 * (warp & 3) + lane, kw0 = (warp - 8) >> 2;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    int i = 0;
    unsigned gc = 0;
    for (int w = blockIdx.x; w < nitems; w += gridDim.x) {
      for (int g = 0; g < G; ++g, ++gc) {
        const int s = g / kGPS, gs = g - s * kGPS;
        const int st = (i + s) % kNS;
        const int b = buf(gc);
        if (gc >= kNB) g_mbar_wait(mmab(b), par(gc - kNB), p.err);   // A buffer b is free
        tc_after();                                     // the stores below come after that MMA's reads
        if (gs == 0) g_mbar_wait(full(st), (unsigned)((i + s) / kNS) & 1u, p.err);
        const unsigned char* stg = ring + (size_t)st * kStage;
        // bf16(128 + q), value j and j + 8 of a word paired in one register: 8 TMEM columns per word
#pragma unroll
        for (int j = 0; j < kWordRows / 2; ++j) {
          const int kw = kw0 + 2 * j;
          uint32_t wd;
          if constexpr (kGU)
            wd = *reinterpret_cast<const uint32_t*>(stg + ((r & 63) >> 5) * 4096 + (gs * 8 + kw) * 256 +
                                                    (r >> 6) * 128 + (r & 31) * 4);
          else
            wd = *reinterpret_cast<const uint32_t*>(stg + (r >> 5) * 4096 + (gs * 8 + kw) * 128 + (r & 31) * 4);
          uint32_t m[8];
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) m[jj] = ((wd >> (2 * jj)) & 0x00030003u) | 0x43004300u;
          asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};\n" ::"r"(
                           tmem + lane_base + (uint32_t)(b * kAcols + kw * 8)),
                       "r"(m[0]), "r"(m[1]), "r"(m[2]), "r"(m[3]), "r"(m[4]), "r"(m[5]), "r"(m[6]), "r"(m[7])
                       : "memory");
        }
        asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
        tc_before();
        g_mbar_arrive(ready(b));
        if (gs == kGPS - 1 || g == G - 1) g_mbar_arrive(empty(st));     // this thread is done with the stage
      }
      i += nsteps;
    }
  }
  // compute warps and the MMA warp: every accumulator was read after its MMA completed (the folds waited on
  // them), so the tensor memory can go
  tc_before();
  asm volatile("bar.sync 3, %0;\n" ::"n"(kCompute + 32 * kMmaWarps) : "memory");
  if (warp == 0) {
    tc_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// y[m, c] = routed_scaling * sum over the token's live routed rows (routing order) of y rows.
__global__ void sum_kernel(const float* yrows, const int32_t* ids, const int32_t* slots, int E, int S, int M, int H,
                           int top_k, float rsf, __nv_bfloat16* y) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)M * H) return;
  const int m = (int)(idx / H), c = (int)(idx - (int64_t)m * H);
  float a = 0.f;
  for (int j = 0; j < top_k; ++j) {
    const int r = m * top_k + j, e = ids[r];
    if (e < 0 || e >= E) continue;
    const int sl = slots[e];
    if (sl >= 0 && sl < S) a += yrows[(int64_t)r * H + c];
  }
  y[idx] = __float2bfloat16(a * rsf);
}

int chunk_tokens(int M, int top_k) {
  int c = kMaxGroupedRows / top_k;
  if (c > kGroupedChunk) c = kGroupedChunk;
  return M < c ? M : c;
}
size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

}  // namespace

// Workspace of the grouped path: the per-token layer's persistent head first (its barrier words and epoch-tagged
// hand-off words must survive calls of either path, so this path never writes there), then for one launch of
// up to chunk_tokens() tokens the route tables, h [R, I] bf16 and the y rows [R, H] fp32.
size_t grouped_workspace_bytes(int M, int H, int I, int top_k) {
  if (M <= 0 || top_k <= 0 || top_k > kMaxGroupedRows) return 0;
  const size_t R = (size_t)chunk_tokens(M, top_k) * top_k;
  return align256(layer_workspace_bytes(0, H, I, top_k)) + align256((16 + 4 * R) * 4) + align256(R * I * 2) +
         align256(R * H * 4);
}

int grouped_check(const LayerArgs& a) {
  if (a.M < kGroupedMinTokens || a.top_k <= 0 || a.top_k > kMaxGroupedRows) return kErrShape;
  if (a.map13.slots == nullptr || a.map13.slots != a.map2.slots || a.map13.E != a.map2.E) return kErrShape;
  if (a.H % kTileCols != 0 || a.I % 64 != 0) return kErrShape;
  if (reinterpret_cast<uintptr_t>(a.x) & 15u) return kErrAlign;
  if (a.workspace == nullptr || a.workspace_bytes < grouped_workspace_bytes(a.M, a.H, a.I, a.top_k))
    return kErrWorkspace;
  if (reinterpret_cast<uintptr_t>(a.workspace) & 255u) return kErrAlign;
  return kOk;
}

int decode_layer_grouped(const LayerArgs& a) {
  CUtensorMap tm[6];
  if (!layer_arena_maps(a, tm)) return kErrShape;
  static thread_local int cached_dev = -1, sms = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kErrDevice;
  if (dev != cached_dev) {
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return kErrDevice;
    if (cudaFuncSetAttribute(proj_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, proj_smem(true)) !=
            cudaSuccess ||
        cudaFuncSetAttribute(proj_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, proj_smem(false)) !=
            cudaSuccess)
      return kErrLaunch;
    cached_dev = dev;
  }
  const int mc_max = chunk_tokens(a.M, a.top_k);
  const int Rmax = mc_max * a.top_k;
  unsigned char* ws = static_cast<unsigned char*>(a.workspace) + align256(layer_workspace_bytes(0, a.H, a.I, a.top_k));
  int* route = reinterpret_cast<int*>(ws);
  __nv_bfloat16* hbuf = reinterpret_cast<__nv_bfloat16*>(ws + align256((16 + 4 * (size_t)Rmax) * 4));
  float* yrows = reinterpret_cast<float*>(ws + align256((16 + 4 * (size_t)Rmax) * 4) +
                                          align256((size_t)Rmax * a.I * 2));
  const bool hz = a.map13.has_zeros != 0;
  for (int m0 = 0; m0 < a.M; m0 += mc_max) {
    const int mc = a.M - m0 < mc_max ? a.M - m0 : mc_max;
    const int R = mc * a.top_k;
    const int32_t* ids = a.ids + (size_t)m0 * a.top_k;
    route_kernel<<<1, 1024, 0, a.stream>>>(ids, a.map13.slots, a.map13.E, a.map13.S, R, route, a.err);
    ProjParams gu{};
    gu.tm[0] = tm[0]; gu.tm[1] = tm[1]; gu.tm[2] = tm[2];
    gu.route = route; gu.R = R;
    gu.act = static_cast<const __nv_bfloat16*>(a.x) + (size_t)m0 * a.H;
    gu.act_stride = a.H; gu.act_row_div = a.top_k;
    gu.K = a.H; gu.N = 2 * a.I; gu.I = a.I;
    gu.has_zeros = hz; gu.scale_bf16 = a.scale_bf16;
    gu.hout = hbuf; gu.err = a.err;
    proj_kernel<true><<<sms, kGThreads, proj_smem(true), a.stream>>>(gu);
    ProjParams dn{};
    dn.tm[0] = tm[3]; dn.tm[1] = tm[4]; dn.tm[2] = tm[5];
    dn.route = route; dn.R = R;
    dn.act = hbuf; dn.act_stride = a.I; dn.act_row_div = 1;
    dn.K = a.I; dn.N = a.H; dn.I = a.I;
    dn.has_zeros = hz; dn.scale_bf16 = a.scale_bf16;
    dn.topk_w = a.topk_w + (size_t)m0 * a.top_k; dn.yrows = yrows; dn.err = a.err;
    proj_kernel<false><<<sms, kGThreads, proj_smem(false), a.stream>>>(dn);
    const int64_t n = (int64_t)mc * a.H;
    sum_kernel<<<(unsigned)((n + 255) / 256), 256, 0, a.stream>>>(yrows, ids, a.map13.slots, a.map13.E, a.map13.S, mc, a.H,
                                                                  a.top_k, a.routed_scaling,
                                                                  static_cast<__nv_bfloat16*>(a.y) + (size_t)m0 * a.H);
    if (cudaGetLastError() != cudaSuccess) return kErrLaunch;
  }
  return kOk;
}

}  // namespace w2a16
