// Batched decode MoE layer (M >= 16 tokens) on the 5th-generation tensor cores (sm_100a tcgen05): the routed
// rows are grouped by expert, so each resident expert's weights cross HBM once per call however many of the
// tokens route to it (the per-token fused layer streams an expert once per routed row). Same computation as
// the composite of patches/ncontig_gemv.py:218-238: gate_up GEMV, SiLU*mul, down GEMV * routed weight,
// top-k sum, with the slot-table indirection of row_arena.py.
//
// route_kernel (one CTA): the live routed rows (slot >= 0) sorted by (slot, row) and cut into groups of at
// most kGN rows of one expert. xtab_kernel: the activation tables (below).
//
// proj_kernel<kGateUp> (persistent, one CTA per SM): work items (group, tile of 128 weight columns -- gate_up:
// 64 gate columns and the matching 64 up columns; down: 128 output columns), dealt round-robin. A producer warp
// streams each item's codes, scales and zero points through a ring of shared-memory stages with tensor copies
// (the fused layer's arena maps). Per 128-value quantization group along K the group's exact integer sums
// come from the tensor cores (kind::i8, int32 accumulation), with the arithmetic of the per-token kernels:
//   * the expansion warps write the codes themselves as the A operand (s8, 0..3) into tensor memory -- one
//     shift and one mask per four codes (the tile's column r is TMEM lane r) -- and the group's scales and
//     zero points into shared memory;
//   * the staging warps copy each routed row's group of the activation table into the B operand (s8,
//     K-major, no swizzle): row n holds token n's high bytes, row 16 + n its low bytes; plus the row's scale
//     and sum. xtab_kernel builds the tables once per call (x) and once between the projections (h): every
//     row's 128 values of a group in 15-bit fixed point with one power-of-two scale, split into a signed high
//     and a signed low byte (x16 = 256 hi + lo), in the K order of the A operand;
//   * an MMA thread (two MMA warps take alternate groups) issues 4 tcgen05.mma (A from tensor memory, M = 128
//     columns, N = 32, K = 32) per group into the group's own accumulator in tensor memory;
//   * two fold sets (taking alternate groups) read the accumulator (tcgen05.ld) and fold it exactly as the
//     reference folds its zero point (gemv/moe_gemv_int2_tab.py:61-66): T = 256 D_hi + D_lo - zp sum x16
//     (exact int32), acc += T * s * 2^e in fp32; at the end of an item the sets add their partial sums and
//     write gate_up -> h = silu(gate) * up in bf16 per routed row, or down -> routed weight * y row in fp32.
// Expansion and staging also come in two sets taking alternate groups. kNB operand/accumulator buffers
// rotate between groups, handed over with mbarriers (operands ready, MMA done, buffer read). Within each
// 16-value word the MMA's K order is the 4 x 4 transpose of the code order (K position p holds code
// 4 * (p % 4) + p / 4); the B operand is staged in the same order.
//
// sum_kernel: y[m] = routed_scaling * (sum of the token's live y rows in routing order), deterministic.
#include <climits>
#include <cuda.h>
#include <cudaTypedefs.h>

#include "w2a16_kernels.h"

namespace w2a16 {
namespace {

constexpr int kGN = 16;                          // routed rows of one group (tokens of one expert)
constexpr int kBN = 2 * kGN;                     // MMA N: a high-byte and a low-byte row per routed row
constexpr int kTileCols = 128;                   // MMA M: weight columns of a tile
constexpr int kSets = 2;                         // fold, expansion and staging sets (4 warps each)
constexpr int kMmaWarps = 2;                     // MMA issuers
// warps: 0-7 fold sets, 8-15 expansion sets, 16-23 staging sets, 24-25 MMA issuers, the producer warp. Set k of
// a role takes the groups gc with gc % kSets == k, MMA warp m those with gc % kMmaWarps == m, so several groups
// are in every stage of the hand-over at once
constexpr int kExpWarp0 = 4 * kSets, kStgWarp0 = 8 * kSets, kMmaWarp0 = 12 * kSets,
              kProducerWarp = kMmaWarp0 + kMmaWarps;
constexpr int kGThreads = 32 * (kProducerWarp + 1);
constexpr int kAcols = kGroup / 4;               // TMEM columns of one group of the A operand (4 codes each)
constexpr int kDcols = kBN;                      // TMEM columns of one group's accumulator
constexpr int kBBytes = kBN * kGroup;            // one group of the B operand (s8)
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
constexpr unsigned kGSpin = 1u << 26;            // mbarrier polls before a spin gives up (well over a second)
constexpr int kNB = 8;                           // operand / accumulator buffers in flight
constexpr int kTmemCols = 512;                   // A: kNB x kAcols columns, then kNB accumulators of kDcols
static_assert(kNB * (kAcols + kDcols) <= kTmemCols, "tensor memory");
// kind::i8 instruction descriptor: s32 accumulator, A and B s8 (the codes 0..3 are non-negative s8), both
// K-major, N = 32, M = 128
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) |
                            ((uint32_t)(kTileCols >> 4) << 24);

__host__ __device__ constexpr int ring_bytes(bool gu) { return gu ? kGURing * kGUStage : kDNRing * kDNStage; }
// per buffer: scales sc[128] f32, zero points zc[128] i32, row scales xe[16] f32, row sums xs[16] i32
constexpr int kSideBytes = kTileCols * 8 + kGN * 8;
// mbarriers (full, empty per stage; ready, mma, free per buffer), tensor-memory address, the fold sets' item
// exchange [128][kGN] and gate_up's up-half exchange [64][kGN]
__host__ __device__ constexpr int small_bytes(bool gu) {
  return (2 * (gu ? kGURing : kDNRing) + 3 * kNB) * 8 + 16 + kTileCols * kGN * 4 + 64 * kGN * 4;
}
__host__ __device__ constexpr int proj_smem(bool gu) {
  return kNB * kBBytes + ring_bytes(gu) + kNB * kSideBytes + small_bytes(gu);
}

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
  const unsigned char* tab;   // activation tables (xtab_kernel): gate_up x rows, down h rows
  const float* xe;            // [rows][G] power-of-two scale of each row and group
  const int* xs;              // [rows][G] sum of the row's 15-bit values over the group
  int act_row_div;            // routed row r reads table row r / act_row_div
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
// Bounded waits for the phase of the given parity (error bit 1 when they give up): suspending tries for the many
// threads of a role, non-suspending polls for the MMA threads (a thread suspended in try_wait resumes some
// time after the phase completes, and the MMA threads' waits are on the hand-over chain of every group).
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
__device__ __forceinline__ void g_mbar_spin(uint32_t bar, unsigned parity, unsigned* err) {
  for (unsigned it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return;
    if (it > kGSpin) {
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
__device__ __forceinline__ void fold_sync() { asm volatile("bar.sync 2, 128;\n" ::: "memory"); }     // fold set 0
__device__ __forceinline__ void fold_sync2() { asm volatile("bar.sync 4, 256;\n" ::: "memory"); }    // both fold sets

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
// One CTA of 1024 threads: the routed rows' (slot, row) keys sorted in shared memory (bitonic; rows whose expert
// is not resident sort last), a group starting at every kGN-th row of one slot, group indices by a block scan.
__global__ void __launch_bounds__(1024) route_kernel(const int32_t* ids, const int32_t* slots, int E, int S, int R,
                                                     int* route, unsigned* err) {
  __shared__ unsigned long long key[kMaxGroupedRows];
  __shared__ int warp_sum[32];
  const RouteView rv{route, R};
  const int t = threadIdx.x;
  {
    unsigned long long kv = ~0ull;                      // padding sorts last
    if (t < R) {
      const int e = ids[t];
      int sl = -1;
      if (e < 0 || e >= E) {
        flag_error(err, 1u);
      } else {
        sl = slots[e];
        if (sl >= S) {                                  // past the arena: masked, flagged
          flag_error(err, 1u);
          sl = -1;
        }
      }
      kv = ((unsigned long long)(sl >= 0 ? (unsigned)sl : 0x7FFFFFFFu) << 32) | (unsigned)t;
    }
    key[t] = kv;
  }
  __syncthreads();
  for (int k = 2; k <= kMaxGroupedRows; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      const int p = t ^ j;
      if (p > t) {
        const unsigned long long a = key[t], b = key[p];
        if ((a > b) == ((t & k) == 0)) {
          key[t] = b;
          key[p] = a;
        }
      }
      __syncthreads();
    }
  // position t of the sorted order: its slot, whether it opens a group (every kGN-th row of a slot's run)
  const bool live = t < R && (unsigned)(key[t] >> 32) != 0x7FFFFFFFu;
  const int k0 = live ? (int)(key[t] >> 32) : -1;
  int first = t;
  if (live)
    while (first > 0 && (int)(key[first - 1] >> 32) == k0) --first;
  const int st = live && (t - first) % kGN == 0 ? 1 : 0;
  // exclusive scan of the group starts: the group index of a starting position
  const int lane = t & 31, w = t >> 5;
  int inc = st;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += v;
  }
  if (lane == 31) warp_sum[w] = inc;
  __syncthreads();
  if (w == 0) {
    int ws = warp_sum[lane], wi = ws;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += v;
    }
    warp_sum[lane] = wi - ws;                           // exclusive prefix of the warp totals
  }
  __syncthreads();
  const int gid = warp_sum[w] + inc - st;
  if (t < R) rv.order()[t] = (int)(unsigned)key[t];
  if (st) {
    int cnt = 1;
    while (t + cnt < R && cnt < kGN && (int)(key[t + cnt] >> 32) == k0) ++cnt;
    rv.gslot()[gid] = k0;
    rv.gstart()[gid] = t;
    rv.gcnt()[gid] = cnt;
  }
  if (t == kMaxGroupedRows - 1) route[0] = warp_sum[w] + inc;   // the number of groups
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
  unsigned char* side = ring + ring_bytes(kGU);       // per buffer: sc, zc, xe, xs
  unsigned char* small = side + kNB * kSideBytes;
  const uint32_t bars = s_u32(small);                 // full[kNS], empty[kNS], ready[kNB], mma[kNB], free[kNB]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(small + (2 * kNS + 3 * kNB) * 8);
  float* part = reinterpret_cast<float*>(small + (2 * kNS + 3 * kNB) * 8 + 16);   // [128][kGN]
  float* upx = part + kTileCols * kGN;                                           // [64][kGN]
  auto sc_of = [&](int b) { return reinterpret_cast<float*>(side + b * kSideBytes); };
  auto zc_of = [&](int b) { return reinterpret_cast<int*>(side + b * kSideBytes + kTileCols * 4); };
  auto xe_of = [&](int b) { return reinterpret_cast<float*>(side + b * kSideBytes + kTileCols * 8); };
  auto xs_of = [&](int b) { return reinterpret_cast<int*>(side + b * kSideBytes + kTileCols * 8 + kGN * 4); };
  auto full = [&](int s) { return bars + 8u * s; };
  auto empty = [&](int s) { return bars + 8u * (kNS + s); };
  auto ready = [&](int b) { return bars + 8u * (2 * kNS + b); };
  auto mmab = [&](int b) { return bars + 8u * (2 * kNS + kNB + b); };
  auto freeb = [&](int b) { return bars + 8u * (2 * kNS + 2 * kNB + b); };
  // group gc uses buffer gc % kNB for the (gc / kNB)-th time: the phase parity of its barriers
  auto buf = [](unsigned gc) { return (int)(gc % kNB); };
  auto par = [](unsigned gc) { return (gc / kNB) & 1u; };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const RouteView rv{p.route, p.R};
  const int G = p.K / kGroup;
  const int nsteps = (G + kGPS - 1) / kGPS;
  const int ntiles = kGU ? p.I / 64 : p.N / kTileCols;
  const bool aligned = (s_u32(smem) & 1023u) == 0;

  if (warp == kProducerWarp && lane == 0) {
    for (int s = 0; s < kNS; ++s) {
      g_mbar_init(full(s), 1);
      g_mbar_init(empty(s), 4 * kGPS);                // per group of the stage, its expansion set's 4 warps
    }
    for (int b = 0; b < kNB; ++b) {
      g_mbar_init(ready(b), 8);                       // the group's expansion set and staging set, 4 warps each
      g_mbar_init(mmab(b), 1);
      g_mbar_init(freeb(b), 4);                       // the group's fold set
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
  const uint32_t tacc = tmem + (uint32_t)(kNB * kAcols);   // accumulator of buffer b at column tacc + b * kDcols
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

  if (warp >= kMmaWarp0) {
    // MMA issuers: per group, once its operands are in place, 4 MMAs of K = 32 into the group's accumulator,
    // committed to the buffer's MMA barrier (the fold set waits on it)
    if (lane == 0) {
      const unsigned m = (unsigned)(warp - kMmaWarp0);
      unsigned gc = 0;
      for (int w = blockIdx.x; w < nitems; w += gridDim.x)
        for (int g = 0; g < G; ++g, ++gc) {
          if (gc % kMmaWarps != m) continue;
          const int b = buf(gc);
          g_mbar_spin(ready(b), par(gc), p.err);
          tc_after();
          const uint64_t bd = kmajor_desc(s_u32(bbuf + b * kBBytes));
          const uint32_t at = tmem + (uint32_t)(b * kAcols), dt = tacc + (uint32_t)(b * kDcols);
          asm volatile("tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, 0;\n" ::"r"(dt), "r"(at), "l"(bd),
                       "r"(kIdesc)
                       : "memory");
#pragma unroll
          for (int k32 = 1; k32 < kGroup / 32; ++k32)   // K slice k32: 8 TMEM columns, 1024 B of B (64 descriptor units)
            asm volatile("tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, 1;\n" ::"r"(dt), "r"(at + 8u * k32),
                         "l"(bd + 64ull * k32), "r"(kIdesc)
                         : "memory");
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(mmab(b))
                       : "memory");
        }
    }
    __syncwarp();
  } else if (warp < kExpWarp0) {
    // ---------------------------------------------------------------- fold sets: thread = tile column r
    const int set = warp >> 2;
    const int r = 32 * (warp & 3) + lane;
    unsigned gc0 = 0;
    for (int w = blockIdx.x; w < nitems; w += gridDim.x, gc0 += (unsigned)G) {
      const int gi = w / ntiles, t = w - gi * ntiles;
      float acc[kGN];
#pragma unroll
      for (int n = 0; n < kGN; ++n) acc[n] = 0.f;
      const int gfirst = (int)(((unsigned)set + kSets - gc0 % kSets) % kSets);
      for (int g = gfirst; g < G; g += kSets) {
        const unsigned gc = gc0 + (unsigned)g;
        const int b = buf(gc);
        g_mbar_wait(ready(b), par(gc), p.err);          // the group's scales, zero points, row scales and sums
        g_mbar_wait(mmab(b), par(gc), p.err);           // and its MMAs are done
        tc_after();
        uint32_t d[kBN];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
            "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]), "=r"(d[7]),
              "=r"(d[8]), "=r"(d[9]), "=r"(d[10]), "=r"(d[11]), "=r"(d[12]), "=r"(d[13]), "=r"(d[14]), "=r"(d[15]),
              "=r"(d[16]), "=r"(d[17]), "=r"(d[18]), "=r"(d[19]), "=r"(d[20]), "=r"(d[21]), "=r"(d[22]), "=r"(d[23]),
              "=r"(d[24]), "=r"(d[25]), "=r"(d[26]), "=r"(d[27]), "=r"(d[28]), "=r"(d[29]), "=r"(d[30]), "=r"(d[31])
            : "r"(tacc + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(b * kDcols)));
        asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
        const float s = sc_of(b)[r];
        const int zp = zc_of(b)[r];
        const float* xe = xe_of(b);
        const int* xs = xs_of(b);
#pragma unroll
        for (int n = 0; n < kGN; ++n) {
          const int T = (int)d[n] * 256 + (int)d[kGN + n] - zp * xs[n];   // exact: |T| < 2^24
          acc[n] = fmaf((float)T, s * xe[n], acc[n]);
        }
        tc_before();
        __syncwarp();
        if (lane == 0) g_mbar_arrive(freeb(b));          // the buffer's accumulator and side data are read
      }
      // the two sets' partial sums of the item, added in set order, then the epilogue by set 0
      if (set == 1)
#pragma unroll
        for (int n = 0; n < kGN; ++n) part[r * kGN + n] = acc[n];
      fold_sync2();
      if (set == 0) {
#pragma unroll
        for (int n = 0; n < kGN; ++n) acc[n] += part[r * kGN + n];
        const int g0 = rv.gstart()[gi], cnt = rv.gcnt()[gi];
        if constexpr (kGU) {
          // rows 0-63 gate, 64-127 up of the tile's 64 h-columns: h = silu(gate) * up
          if (r >= 64)
#pragma unroll
            for (int n = 0; n < kGN; ++n) upx[(r - 64) * kGN + n] = acc[n];
          fold_sync();
          if (r < 64)
#pragma unroll
            for (int n = 0; n < kGN; ++n)
              if (n < cnt) {
                const int row = rv.order()[g0 + n];
                p.hout[(int64_t)row * p.I + 64 * t + r] = __float2bfloat16(silu(acc[n]) * upx[r * kGN + n]);
              }
          fold_sync();
        } else {
#pragma unroll
          for (int n = 0; n < kGN; ++n)
            if (n < cnt) {
              const int row = rv.order()[g0 + n];
              p.yrows[(int64_t)row * p.N + kTileCols * t + r] = p.topk_w[row] * acc[n];
            }
        }
      }
      fold_sync2();                                     // set 0 has read the exchange before set 1 writes again
    }
  } else if (warp >= kStgWarp0) {
    // ---------------------------------------------------------------- staging sets: the B operand
    // thread: routed row bn of the group (B rows bn and kGN + bn), 16-value word bs of each group; a set's table
    // pieces of its next two groups are in flight while it stores one
    const int set = (warp - kStgWarp0) >> 2;
    const int r = tid - 32 * (kStgWarp0 + 4 * set);
    const int bn = r >> 3, bs = r & 7;
    unsigned gc0 = 0;
    struct Piece { uint4 h, l; float e; int s; };
    for (int w = blockIdx.x; w < nitems; w += gridDim.x, gc0 += (unsigned)G) {
      const int gi = w / ntiles;
      const int g0 = rv.gstart()[gi], cnt = rv.gcnt()[gi];
      const int trow = bn < cnt ? rv.order()[g0 + bn] / p.act_row_div : -1;   // table row, -1 = padding
      const int gfirst = (int)(((unsigned)set + kSets - gc0 % kSets) % kSets);
      auto fetch = [&](int g, Piece& pc) {
        pc.h = pc.l = make_uint4(0, 0, 0, 0);
        pc.e = 0.f;
        pc.s = 0;
        if (trow < 0 || g >= G) return;
        const unsigned char* src = p.tab + ((size_t)trow * G + g) * 256 + bs * 16;
        pc.h = *reinterpret_cast<const uint4*>(src);
        pc.l = *reinterpret_cast<const uint4*>(src + 128);
        if (bs == 0) {
          pc.e = p.xe[(size_t)trow * G + g];
          pc.s = p.xs[(size_t)trow * G + g];
        }
      };
      auto store = [&](int g, const Piece& pc) {
        const unsigned gc = gc0 + (unsigned)g;
        const int b = buf(gc);
        if (gc >= kNB) g_mbar_wait(freeb(b), par(gc - kNB), p.err);   // buffer b's previous group is folded
        unsigned char* B = bbuf + b * kBBytes + (bs >> 1) * 1024;
        *reinterpret_cast<uint4*>(B + canon_off(bn, bs & 1)) = pc.h;
        *reinterpret_cast<uint4*>(B + canon_off(kGN + bn, bs & 1)) = pc.l;
        if (bs == 0) {
          xe_of(b)[bn] = pc.e;
          xs_of(b)[bn] = pc.s;
        }
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");   // generic writes -> the MMA's reads
        __syncwarp();
        if (lane == 0) g_mbar_arrive(ready(b));
      };
      constexpr int kStep = kSets;
      Piece pa, pb;
      fetch(gfirst, pa);
      fetch(gfirst + kStep, pb);
      for (int g = gfirst; g < G; g += 2 * kStep) {
        store(g, pa);
        fetch(g + 2 * kStep, pa);
        if (g + kStep < G) {
          store(g + kStep, pb);
          fetch(g + 3 * kStep, pb);
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- expansion sets: codes -> A in TMEM
    // warp kExpWarp0 + 4 set + q takes TMEM lanes (tile columns) 32 q .. + 31 of its set's groups
    const bool sbf = p.scale_bf16 != 0, hz = p.has_zeros != 0;
    const int set = (warp - kExpWarp0) >> 2;
    const int r = 32 * (warp & 3) + lane;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    int i = 0;                                          // the CTA's stage count at the item's start
    unsigned gc0 = 0;
    for (int w = blockIdx.x; w < nitems; w += gridDim.x, i += nsteps, gc0 += (unsigned)G) {
      const int gfirst = (int)(((unsigned)set + kSets - gc0 % kSets) % kSets);
      for (int g = gfirst; g < G; g += kSets) {
        const unsigned gc = gc0 + (unsigned)g;
        const int s = g / kGPS, gs = g - s * kGPS;
        const int st = (i + s) % kNS;
        const int b = buf(gc);
        if (gc >= kNB) g_mbar_wait(freeb(b), par(gc - kNB), p.err);   // buffer b's previous group is folded
        tc_after();                                     // the stores below come after that group's MMAs
        g_mbar_wait(full(st), (unsigned)((i + s) / kNS) & 1u, p.err);
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
        sc_of(b)[r] = sbf ? __bfloat162float(__ushort_as_bfloat16((unsigned short)raw))
                          : __half2float(__ushort_as_half((unsigned short)raw));
        zc_of(b)[r] = zp;
        // word kw -> 4 TMEM columns: class c = codes c, 4 + c, 8 + c, 12 + c as bytes (bits 2c of each byte)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t m[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int kw = 4 * h + j;
            uint32_t wd;
            if constexpr (kGU)
              wd = *reinterpret_cast<const uint32_t*>(stg + ((r & 63) >> 5) * 4096 + (gs * 8 + kw) * 256 +
                                                      (r >> 6) * 128 + (r & 31) * 4);
            else
              wd = *reinterpret_cast<const uint32_t*>(stg + (r >> 5) * 4096 + (gs * 8 + kw) * 128 + (r & 31) * 4);
#pragma unroll
            for (int c = 0; c < 4; ++c) m[4 * j + c] = (wd >> (2 * c)) & 0x03030303u;
          }
          asm volatile(
              "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
              "%14, %15, %16};\n" ::"r"(tmem + lane_base + (uint32_t)(b * kAcols + 16 * h)),
              "r"(m[0]), "r"(m[1]), "r"(m[2]), "r"(m[3]), "r"(m[4]), "r"(m[5]), "r"(m[6]), "r"(m[7]), "r"(m[8]),
              "r"(m[9]), "r"(m[10]), "r"(m[11]), "r"(m[12]), "r"(m[13]), "r"(m[14]), "r"(m[15])
              : "memory");
        }
        asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
        tc_before();
        __syncwarp();                                   // the warp's stores are complete and its stage reads done
        if (lane == 0) {
          g_mbar_arrive(ready(b));
          // the stage's empty barrier counts 4 arrivals per group; the last group of an item also stands in for
          // the groups a short last stage lacks
          g_mbar_arrive(empty(st));
          if (g == G - 1)
            for (int k = gs + 1; k < kGPS; ++k) g_mbar_arrive(empty(st));
        }
      }
    }
  }
  // all but the producer: every group's MMAs completed before its fold set read the accumulator, so the tensor
  // memory can go
  tc_before();
  asm volatile("bar.sync 3, %0;\n" ::"n"(kGThreads - 32) : "memory");
  if (warp == 0) {
    tc_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// Activation tables for the B operand: rows x K bf16 -> per (row, 128-value group) 256 bytes (8 words x 16 high
// bytes, then 8 words x 16 low bytes; K position 4c + j of a word holds value 4j + c), the power-of-two scale
// 2^(e - 14) (mx = f 2^e, f in [0.5, 1), so |x16| <= 2^14) and the sum of the 128 values x16. Eight lanes per
// (row, group), one 16-value word each.
__global__ void __launch_bounds__(256) xtab_kernel(const __nv_bfloat16* act, int rows, int64_t stride, int G,
                                                   unsigned char* tab, float* xe, int* xs) {
  const int team = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 3);
  const int bs = threadIdx.x & 7;
  const bool live = team < rows * G;
  const int row = live ? team / G : 0, g = live ? team - row * G : 0;
  float v[16];
  {
    uint4 pa = make_uint4(0, 0, 0, 0), pb = pa;
    if (live) {
      const __nv_bfloat16* src = act + (int64_t)row * stride + g * kGroup + bs * 16;
      pa = *reinterpret_cast<const uint4*>(src);
      pb = *reinterpret_cast<const uint4*>(src + 8);
    }
    const uint32_t u[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      v[2 * k] = __uint_as_float(u[k] << 16);
      v[2 * k + 1] = __uint_as_float(u[k] & 0xFFFF0000u);
    }
  }
  float mx = 0.f;
#pragma unroll
  for (int k = 0; k < 16; ++k) mx = fmaxf(mx, fabsf(v[k]));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
  const int e = mx > 0.f ? frexp_exponent(mx) : 0;
  const float inv = pow2f(14 - e);
  // t = x16 + 128: its byte 1 is the signed high byte hi = (x16 + 128) >> 8, its byte 0 xor 0x80 the signed
  // low byte lo = x16 - 256 hi
  uint32_t t[16];
  int sum = 0;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const int q = __float2int_rn(v[k] * inv);
    sum += q;
    t[k] = (uint32_t)(q + 128);
  }
  sum += __shfl_xor_sync(0xffffffffu, sum, 1);
  sum += __shfl_xor_sync(0xffffffffu, sum, 2);
  sum += __shfl_xor_sync(0xffffffffu, sum, 4);
  uint32_t H[4], L[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    // values c, 4 + c, 8 + c, 12 + c -> bytes 0..3
    H[c] = __byte_perm(__byte_perm(t[c], t[4 + c], 0x0051), __byte_perm(t[8 + c], t[12 + c], 0x0051), 0x5410);
    L[c] = __byte_perm(__byte_perm(t[c], t[4 + c], 0x0040), __byte_perm(t[8 + c], t[12 + c], 0x0040), 0x5410) ^
           0x80808080u;
  }
  if (!live) return;
  unsigned char* dst = tab + (size_t)team * 256 + bs * 16;
  *reinterpret_cast<uint4*>(dst) = make_uint4(H[0], H[1], H[2], H[3]);
  *reinterpret_cast<uint4*>(dst + 128) = make_uint4(L[0], L[1], L[2], L[3]);
  if (bs == 0) {
    xe[team] = pow2f(e - 14);
    xs[team] = sum;
  }
}

// y[m, c] = routed_scaling * sum over the token's live routed rows (routing order) of y rows. One CTA per token:
// the token's rows are resolved once into shared memory.
__global__ void __launch_bounds__(256) sum_kernel(const float* yrows, const int32_t* ids, const int32_t* slots, int E,
                                                  int S, int M, int H, int top_k, float rsf, __nv_bfloat16* y) {
  __shared__ int live_rows[kMaxGroupedRows];
  __shared__ int nlive;
  const int m = blockIdx.x;
  if (threadIdx.x == 0) {
    int n = 0;
    for (int j = 0; j < top_k; ++j) {
      const int r = m * top_k + j, e = ids[r];
      if (e < 0 || e >= E) continue;
      const int sl = slots[e];
      if (sl >= 0 && sl < S) live_rows[n++] = r;
    }
    nlive = n;
  }
  __syncthreads();
  const int n = nlive;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float a = 0.f;
    for (int j = 0; j < n; ++j) a += yrows[(int64_t)live_rows[j] * H + c];
    y[(int64_t)m * H + c] = __float2bfloat16(a * rsf);
  }
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
// Bytes of the activation tables of `rows` rows of K values (xtab_kernel): 256 per (row, group), then the scales
// and the sums.
size_t tab_bytes(size_t rows, int K) {
  const size_t n = rows * (size_t)(K / kGroup);
  return align256(n * 256) + align256(n * 4) + align256(n * 4);
}
size_t grouped_workspace_bytes(int M, int H, int I, int top_k) {
  if (M <= 0 || top_k <= 0 || top_k > kMaxGroupedRows) return 0;
  const size_t mc = (size_t)chunk_tokens(M, top_k), R = mc * top_k;
  return align256(layer_workspace_bytes(0, H, I, top_k)) + align256((16 + 4 * R) * 4) + align256(R * I * 2) +
         align256(R * H * 4) + tab_bytes(mc, H) + tab_bytes(R, I);
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
  // activation tables: x (mc_max rows of H), then h (Rmax rows of I)
  struct Tab { unsigned char* t; float* e; int* s; };
  auto carve = [](unsigned char* base, size_t rows, int K) {
    const size_t n = rows * (size_t)(K / kGroup);
    return Tab{base, reinterpret_cast<float*>(base + align256(n * 256)),
               reinterpret_cast<int*>(base + align256(n * 256) + align256(n * 4))};
  };
  unsigned char* tabs = reinterpret_cast<unsigned char*>(yrows) + align256((size_t)Rmax * a.H * 4);
  const Tab xt = carve(tabs, (size_t)mc_max, a.H);
  const Tab ht = carve(tabs + tab_bytes((size_t)mc_max, a.H), (size_t)Rmax, a.I);
  const int G1 = a.H / kGroup, G2 = a.I / kGroup;
  const bool hz = a.map13.has_zeros != 0;
  for (int m0 = 0; m0 < a.M; m0 += mc_max) {
    const int mc = a.M - m0 < mc_max ? a.M - m0 : mc_max;
    const int R = mc * a.top_k;
    const int32_t* ids = a.ids + (size_t)m0 * a.top_k;
    route_kernel<<<1, 1024, 0, a.stream>>>(ids, a.map13.slots, a.map13.E, a.map13.S, R, route, a.err);
    const int nx = mc * G1 * 8;                         // 8 lanes per (row, group)
    xtab_kernel<<<(unsigned)((nx + 255) / 256), 256, 0, a.stream>>>(
        static_cast<const __nv_bfloat16*>(a.x) + (size_t)m0 * a.H, mc, a.H, G1, xt.t, xt.e, xt.s);
    ProjParams gu{};
    gu.tm[0] = tm[0]; gu.tm[1] = tm[1]; gu.tm[2] = tm[2];
    gu.route = route; gu.R = R;
    gu.tab = xt.t; gu.xe = xt.e; gu.xs = xt.s; gu.act_row_div = a.top_k;
    gu.K = a.H; gu.N = 2 * a.I; gu.I = a.I;
    gu.has_zeros = hz; gu.scale_bf16 = a.scale_bf16;
    gu.hout = hbuf; gu.err = a.err;
    proj_kernel<true><<<sms, kGThreads, proj_smem(true), a.stream>>>(gu);
    const int nh = R * G2 * 8;
    xtab_kernel<<<(unsigned)((nh + 255) / 256), 256, 0, a.stream>>>(hbuf, R, a.I, G2, ht.t, ht.e, ht.s);
    ProjParams dn{};
    dn.tm[0] = tm[3]; dn.tm[1] = tm[4]; dn.tm[2] = tm[5];
    dn.route = route; dn.R = R;
    dn.tab = ht.t; dn.xe = ht.e; dn.xs = ht.s; dn.act_row_div = 1;
    dn.K = a.I; dn.N = a.H; dn.I = a.I;
    dn.has_zeros = hz; dn.scale_bf16 = a.scale_bf16;
    dn.topk_w = a.topk_w + (size_t)m0 * a.top_k; dn.yrows = yrows; dn.err = a.err;
    proj_kernel<false><<<sms, kGThreads, proj_smem(false), a.stream>>>(dn);
    sum_kernel<<<(unsigned)mc, 256, 0, a.stream>>>(yrows, ids, a.map13.slots, a.map13.E, a.map13.S, mc, a.H, a.top_k,
                                                  a.routed_scaling, static_cast<__nv_bfloat16*>(a.y) + (size_t)m0 * a.H);
    if (cudaGetLastError() != cudaSuccess) return kErrLaunch;
  }
  return kOk;
}

}  // namespace w2a16
