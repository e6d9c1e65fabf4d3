// Decode MoE layer in one cooperative kernel: gate_up GEMV + SiLU*mul, down GEMV * routed weight,
// sum over the top-k experts of each token (the composite of patches/ncontig_gemv.py:218-238).
//
// Prologue. The routing (ids -> slot -> expert bases) is resolved first, the activation rows are turned
// into fixed-point tables while those loads are in flight, and one warp compacts the live routed rows
// (slot >= 0) with ballots, so the first weight copy is issued a few hundred nanoseconds after the
// routing arrives.
//
// Phase 1 (gate_up). Work items are (live row r, block of 32 h-columns, 2 groups of K): 32 lanes = 2
// groups x 16 column quads, quads 0-7 over the 32 gate columns and 8-15 over the matching 32 up columns.
// The items are cut into one contiguous range per CTA (sizes differ by at most one, and a range is at
// least one h-block long, so no block spans more than two CTAs); a CTA's 16 warps share its range
// round-robin and leave one 64-float partial per item in shared memory. The CTA then finishes each h-block
// that starts in its range, in item order (deterministic): the tail of a block that runs into the next
// CTA comes from that CTA's published partial sums (neighbour hand-off, bounded wait on its flag).
// A finished block's 32 values h = silu(gate) * up are written straight into the row's down-projection
// activation table in the workspace: 16-bit fixed point with one power-of-two exponent per 32 values
// (the block), so no CTA ever converts h again.
//
// One grid barrier (bounded wait), then phase 2 (down). Work units are (token m, block of 32 output
// columns): live rows x ceil(G2/4) K-parts = items of 4 groups x 8 column quads. Units are dealt
// round-robin to CTAs and processed one at a time: the unit's h tables are bulk-copied into shared
// memory, its items reduced, and its partials summed in fixed order into y. No atomics beyond the
// barrier and the hand-off flags.
//
// Weight stream. Copy-engine mode (slot arenas): producer threads stream every item's codes, scales
// and zero points through a ring of shared-memory stages with tensor copies, phase-2 items right behind
// phase-1 items, so the down weights are in flight while phase 1 finishes. Register mode (int64 address
// tables): at launch every CTA asks L2 to fetch its 1/grid share of each routed expert's arrays, and each
// lane loads its own item data into registers one item ahead of the one it is reducing.
//
// Expert parallelism (the kEx variant; the plain variant carries none of it). With a PeerExchange channel the
// prologue's table warps take x as the sum, in rank order, of the ranks' tagged rows of the channel's call
// (each 8-byte word -- two bf16 values and the call number -- polled until it holds the call), and phase 2
// pushes each finished unit of y as this rank's tagged row of the next call into every rank's buffer instead
// of writing y; the all-reduce of the ranks' partials thereby rides on the layers' own loads and stores.
#include <cuda.h>
#include <type_traits>
#include <cudaTypedefs.h>

#include "w2a16_kernels.h"

namespace w2a16 {
namespace {

constexpr int kThreads = 512;                                // reducing warps (both modes)
constexpr int kWarps = kThreads / 32;
constexpr int kProducers = 4;                                // producer warps (copy-engine mode)
constexpr int kIssuers = 2 * kProducers;                     // issuing threads: lanes 0 and 1 of each
constexpr int kTmaThreads = kThreads + 32 * kProducers;
// Copy-engine mode: one stage of the shared-memory ring holds one item -- codes at 0 (4 KB: 16 word rows
// x [32 gate | 32 up] columns, or 32 word rows x 32 columns), scales at 4096 (256 B), zero-point windows
// at 4352 (64 B); every offset a multiple of 128 bytes, as tensor copies require.
constexpr int kStageBytes = 4480;
constexpr int kScaleOff = 4096;
constexpr int kZeroOff = 4352;
constexpr int kMinStages = 16, kMaxStages = 48;             // multiples of kIssuers

constexpr unsigned kSpinLimit = 1u << 22;                    // polls before a wait gives up
constexpr unsigned kWaitLimit = 1u << 17;                    // suspending mbarrier tries before a wait gives up

// Division of a non-negative int below 2^31 by a divisor d >= 1 fixed at launch: q = (x * m) >> s with
// l = ceil(log2 d), s = 31 + l, m = ceil(2^s / d) < 2^32 -- exact for every such x (the round-up method
// for unsigned division by invariant integers, Granlund and Montgomery 1994).
struct FDiv {
  uint32_t m;
  int s;
};
FDiv make_fdiv(int d) {
  int l = 0;
  while ((1ll << l) < d) ++l;
  const int s = 31 + l;
  return FDiv{(uint32_t)(((1ull << s) + (uint64_t)d - 1) / (uint64_t)d), s};
}
__device__ __forceinline__ int fdiv(int x, FDiv d) {
  return (int)(((uint64_t)(uint32_t)x * d.m) >> d.s);
}

struct Geo {
  int M, H, I, top_k, R;
  int G1, G2;          // groups along K of gate_up (H/128) and down (I/128)
  int nb1, kp1;        // h-blocks per row (I/32), items per h-block (ceil(G1/2))
  int nb2, kp2;        // output blocks per token (H/32), K-parts per row (ceil(G2/4))
  int n1;              // phase-1 items
  int u2, s2;          // phase-2 units (M * nb2), items per unit (top_k * kp2)
  int grid;            // CTAs
  int max_range;       // max phase-1 items per CTA
  int max_units;       // max phase-2 units per CTA
  FDiv d_kp1, d_nb1, d_row1, d_kp2, d_nb2, d_s2, d_topk, d_G1;   // row1 = nb1 * kp1 (items per row)
  int stab;            // slot-table entries staged in shared memory (0: looked up in global memory)
};

Geo make_geo(int M, int H, int I, int top_k, int grid_cap) {
  Geo g{};
  g.M = M; g.H = H; g.I = I; g.top_k = top_k; g.R = M * top_k;
  g.G1 = H / kGroup; g.G2 = I / kGroup;
  g.nb1 = I / 32; g.kp1 = (g.G1 + 1) / 2;
  g.nb2 = H / 32; g.kp2 = (g.G2 + 3) / 4;
  g.n1 = g.R * g.nb1 * g.kp1;
  g.u2 = M * g.nb2; g.s2 = top_k * g.kp2;
  const int nblocks = g.R * g.nb1;                  // a CTA range must cover at least one h-block
  g.grid = grid_cap < nblocks ? grid_cap : nblocks;
  if (g.grid < 1) g.grid = 1;
  g.max_range = (g.n1 + g.grid - 1) / g.grid;
  g.max_units = (g.u2 + g.grid - 1) / g.grid;
  g.d_kp1 = make_fdiv(g.kp1); g.d_nb1 = make_fdiv(g.nb1); g.d_row1 = make_fdiv(g.nb1 * g.kp1);
  g.d_kp2 = make_fdiv(g.kp2); g.d_nb2 = make_fdiv(g.nb2); g.d_s2 = make_fdiv(g.s2);
  g.d_topk = make_fdiv(top_k); g.d_G1 = make_fdiv(g.G1);
  return g;
}

__host__ __device__ __forceinline__ size_t token_table_bytes(int K) {
  return ((size_t)(K / 16) * kXRegs * 4 + (size_t)(K / kGroup) * 8 + 15) & ~size_t(15);
}

// Down-projection activation table of one routed row (K = I): packed pairs [I/16][kXRegs], then per
// 32-value sub-group m64x [I/32] and scl [I/32]. I is a multiple of 128, so the size is a multiple of
// 16 bytes and rows can be moved with bulk copies.
constexpr int kSub = 32;                                     // values per exponent in the h tables
__host__ __device__ __forceinline__ size_t htab_bytes(int I) {
  return (size_t)(I / 16) * kXRegs * 4 + (size_t)(I / kSub) * 8;
}

struct SmemPlan {
  size_t tabs, mail1, mail2, rows, misc, live, slots, preg, total;
};
constexpr int kMaxStagedSlots = 2048;                        // slot tables up to 8 KB are staged
constexpr int kMaxPrivSlots = 512;                           // producers keep private copies up to 2 KB

// Copy-engine producers route privately (no hand-over from warp 0) when the routed rows fit one warp and
// the slot table is staged and small: region per producer warp = slot, rowmap, tokrow, tokcnt [32 each]
// and the slot table.
__host__ __device__ __forceinline__ bool private_routing(const Geo& g) {
  return g.R <= 32 && g.stab > 0 && g.stab <= kMaxPrivSlots;
}
__host__ __device__ __forceinline__ int preg_ints(const Geo& g) { return (128 + g.stab + 3) & ~3; }

// Per routed row, resolved once per CTA: expert code / scale / zero-point bases of gate_up and down.
struct RowPtr {
  const uint32_t* w[2];
  const char* s[2];
  const uint8_t* z[2];
  int ok[2];
  int slot;      // arena slot of the row's expert (copy-engine mode)
  float wt;      // routing weight
};

SmemPlan smem_plan(const Geo& g) {
  SmemPlan s{};
  const size_t t1 = (size_t)g.M * token_table_bytes(g.H);
  const size_t t2 = (size_t)g.top_k * htab_bytes(g.I);         // one down unit's h tables at a time
  s.tabs = t1 > t2 ? t1 : t2;
  s.mail1 = (size_t)g.max_range * 64 * 4;
  s.mail2 = (size_t)g.s2 * 32 * 4;
  s.rows = ((size_t)g.R * sizeof(RowPtr) + 15) & ~size_t(15);
  s.misc = 64;                                                  // mbarrier, head counter, generation
  // LiveRows arrays and the live-row bit words
  s.live = ((size_t)(2 * g.R + g.M + g.max_units * g.top_k + (g.R + 31) / 32) * 4 + 15) & ~size_t(15);
  s.slots = ((size_t)g.stab * 4 + 15) & ~size_t(15);
  s.preg = private_routing(g) ? (size_t)kProducers * preg_ints(g) * 4 : 0;   // (copy-engine mode only)
  s.total = s.tabs + s.mail1 + s.mail2 + s.rows + s.misc + s.live + s.slots + s.preg;
  return s;
}

struct FusedParams {
  // copy-engine mode: tensor maps over the slot arena -- gate_up codes / scales / zero points (4-D:
  // column within half, half, row, slot) and down codes / scales / zero points (3-D: column, row, slot)
  CUtensorMap tm[6];
  int nstage;
  size_t off_stages, off_bars;
  const __nv_bfloat16* x;
  const int32_t* ids;
  const float* topk_w;
  ExpertMap map13, map2;
  int scale_bf16;
  float rsf;
  __nv_bfloat16* y;
  Geo geo;
  size_t off_tabs, off_mail1, off_mail2, off_rows, off_misc, off_live, off_slots, off_preg;
  unsigned* bar_count;   // grid barrier: arrivals (zero between calls)
  unsigned* bar_gen;     // grid barrier: generation, 128 bytes further
  unsigned char* htab;   // [R][htab_bytes(I)] down-projection activation tables of the routed rows
  // [grid][2 (gate, up)][32 columns] hand-off words: (epoch << 32) | float bits of the partial sums a CTA
  // publishes for the tail of the h-block it shares with the previous CTA
  unsigned long long* hand;
  unsigned* err;
  // expert parallelism (a PeerExchange channel): xin -- x is the sum of the ranks' rows of the channel's call
  // e = *xepoch; yout -- this layer's partial y goes out as this rank's tagged row of call e + 1 into every
  // rank's buffer, and CTA 0 stores *xepoch = e + 1 when it is done
  int xin, yout;
  const uint64_t* xpeers;
  size_t xtag_off;
  int xn_max, xrank, xworld;
  unsigned* xepoch;
  unsigned xspin;
};

// Activation table of a K-long row: one exponent per 128-value group (gate_up, from x) ...
__device__ __forceinline__ XTable table_at(unsigned char* base, int K) {
  XTable t;
  t.pairs = reinterpret_cast<uint32_t*>(base);
  t.m64x = reinterpret_cast<int*>(base + (size_t)(K / 16) * kXRegs * 4);
  t.scl = reinterpret_cast<float*>(t.m64x + K / kGroup);
  return t;
}
// ... or one per 32-value sub-group (down, from h).
__device__ __forceinline__ XTable htable_at(unsigned char* base, int I) {
  XTable t;
  t.pairs = reinterpret_cast<uint32_t*>(base);
  t.m64x = reinterpret_cast<int*>(base + (size_t)(I / 16) * kXRegs * 4);
  t.scl = reinterpret_cast<float*>(t.m64x + I / kSub);
  return t;
}

// The 32 values of h-block hb (lane l holds element 32*hb + l) -> fixed-point entries of a down table:
// exponent from the block's max |h| exactly as the 128-value activation groups take theirs, values
// rounded to nearest and clamped to +-32767, pairs packed as in the activation tables (elements c and
// c + 4 of a 16-value word row share a register). Whole warp, uniform control flow.
__device__ __forceinline__ void htab_block(unsigned char* tab, int I, int hb, float h, int lane) {
  const float mx = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(h))));
  const int e = (mx > 0.f ? frexp_exponent(mx) : 0) - 15;
  const int q = max(-32767, min(32767, __float2int_rn(h * pow2f(-e))));
  const int s = __reduce_add_sync(0xffffffffu, q);
  const int hi = __shfl_xor_sync(0xffffffffu, q, 4);
  if ((lane & 4) == 0) {
    const int c = lane & 15, kw = hb * 2 + (lane >> 4);
    reinterpret_cast<uint32_t*>(tab)[kw * kXRegs + (c & 3) * 2 + (c >> 3)] = (uint32_t)(q & 0xFFFF) | ((uint32_t)hi << 16);
  }
  if (lane == 0) {
    int* m64x = reinterpret_cast<int*>(tab + (size_t)(I / 16) * kXRegs * 4);
    m64x[hb] = -64 * s;
    reinterpret_cast<float*>(m64x + I / kSub)[hb] = pow2f(e - 6);
  }
}

// One warp copies the first n entries of the slot table into shared memory. Every load of a lane is
// issued before its first store: the compiler cannot tell the two arrays apart, so a store between two
// loads would hold the second back until the first returned (one global round trip per 32 entries).
__device__ __forceinline__ void stage_slots(int* dst, const int* src, int n, int lane) {
  constexpr int kPer = 16;
  for (int k0 = 0; k0 < n; k0 += 32 * kPer) {
    int v[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int k = k0 + lane + 32 * j;
      v[j] = k < n ? src[k] : 0;
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int k = k0 + lane + 32 * j;
      if (k < n) dst[k] = v[j];
    }
  }
}

// Barrier of the 512 reducing threads only (the producer warps of copy-engine mode never join).
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;\n" ::"n"(kThreads) : "memory"); }
// Prologue hand-overs of copy-engine mode: warp 0 -> producer warps once the routing is compacted
// (barrier 2), producer warps -> reducing warps once the ring barriers exist (barrier 3).
__device__ __forceinline__ void bar_arrive(int id, int n) { asm volatile("bar.arrive %0, %1;\n" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ void bar_wait(int id, int n) { asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(n) : "memory"); }


// One entry of a warp's work list.
struct Work {
  int kind;   // 0 none, 1 gate_up, 2 down
  int r, b, kp;
  int slot;   // mailbox index within the CTA
  int unit;   // phase 2: unit slot within the CTA
  int jr;     // phase 2: row index within the token
  int seq;    // position in the CTA's item order (copy-engine ring)
  int dead;   // phase 2: slot past the token's live rows (reduces nothing, writes a zero partial)
};

// Routed rows whose expert resolves (slot >= 0), compacted identically by every CTA in its prologue.
// Phase-1 items and ranges run over the live rows only, so masked rows (experts not resident, or owned
// by another GPU) cost nothing and do not unbalance the CTAs; phase-2 items of a token take its live
// rows first and the remaining (dead) item slots of its units write zero partials.
struct LiveRows {
  const int* rowmap;   // [R] compact phase-1 row -> routed row
  const int* tokrow;   // [M][top_k] j-th live row of token m, as an index within the token's top_k
  const int* tokcnt;   // [M] live rows per token
  const int* slotrow;  // [max_units][top_k] routed row of slot jr of this CTA's unit q, -1 = dead
  int n1;              // phase-1 items over the live rows
  int grid1;           // CTAs holding phase-1 items (each range at least one h-block)
};

struct WarpList {
  int a;      // CTA's phase-1 range start
  int b;      // CTA's phase-1 range end
  int range;  // CTA's phase-1 items
  int n1w;    // phase-1 items of this warp
  int nu;     // phase-2 units of this CTA
  int n2w;    // phase-2 items of this warp per unit
  __device__ int total() const { return n1w + nu * n2w; }
};

// CTA ranges: the first n1 % grid1 CTAs take one item more than the others.
__device__ __forceinline__ WarpList warp_list(const Geo& g, const LiveRows& lv, int cta, int warp) {
  WarpList L;
  L.a = L.b = lv.n1;
  if (cta < lv.grid1) {
    const int q = lv.n1 / lv.grid1, rem = lv.n1 - q * lv.grid1;
    L.a = cta * q + min(cta, rem);
    L.b = L.a + q + (cta < rem ? 1 : 0);
  }
  const int range = L.b - L.a;
  L.range = range;
  L.n1w = range > warp ? (range - warp + kWarps - 1) / kWarps : 0;
  L.nu = cta < g.u2 ? (g.u2 - cta + g.grid - 1) / g.grid : 0;
  L.n2w = g.s2 > warp ? (g.s2 - warp + kWarps - 1) / kWarps : 0;
  return L;
}

// Phase-2 item j of unit (token m, block b) -> its live row (or a dead slot).
__device__ __forceinline__ void unit_row(const Geo& g, const LiveRows& lv, int m, int j, Work& w) {
  w.jr = fdiv(j, g.d_kp2);
  w.kp = j - w.jr * g.kp2;
  w.dead = w.jr >= lv.tokcnt[m];
  w.r = m * g.top_k + (w.dead ? w.jr : lv.tokrow[m * g.top_k + w.jr]);
}

// The warp's t-th gate_up item ...
__device__ __forceinline__ Work work1(const Geo& g, const LiveRows& lv, const WarpList& L, int warp, int t) {
  Work w{};
  const int i = L.a + warp + kWarps * t;
  w.kind = 1;
  const int rc = fdiv(i, g.d_row1);
  w.r = lv.rowmap[rc];
  const int rem = i - rc * (g.nb1 * g.kp1);
  w.b = fdiv(rem, g.d_kp1);
  w.kp = rem - w.b * g.kp1;
  w.slot = i - L.a;
  w.seq = warp + kWarps * t;
  return w;
}

// ... and its k-th down item of unit q.
__device__ __forceinline__ Work work2(const Geo& g, const LiveRows& lv, const WarpList& L, int cta, int warp, int q,
                                     int k) {
  Work w{};
  const int u = cta + g.grid * q, j = warp + kWarps * k;
  const int m = fdiv(u, g.d_nb2);
  w.kind = 2;
  w.b = u - m * g.nb2;
  unit_row(g, lv, m, j, w);
  w.unit = q;
  w.slot = j;                 // mail2 holds one unit at a time
  w.seq = L.range + q * g.s2 + j;
  return w;
}

// Lane -> (group within the item, first of its 4 columns, group index along K). Gate_up items: lanes
// 0-15 take group 2kp, 16-31 group 2kp+1, quads 0-7 over the 32 gate columns and 8-15 over the matching
// up columns. Down items: 4 groups x 8 column quads.
struct LaneMap {
  int col, gl;
  bool valid;
};

template <int kKind>
__device__ __forceinline__ LaneMap lane_map_k(const Geo& g, const Work& w, int lane, const RowPtr* rows) {
  LaneMap lm{};
  if (w.kind != kKind) return lm;
  constexpr bool k1 = kKind == 1;
  const int gi = k1 ? (lane >> 4) : (lane >> 3);
  const int q = k1 ? (lane & 15) : (lane & 7);
  const int q8 = k1 ? (q & 7) : q;
  lm.col = (k1 && q >= 8 ? g.I : 0) + w.b * 32 + q8 * 4;
  lm.gl = k1 ? w.kp * 2 + gi : w.kp * 4 + gi;
  lm.valid = !w.dead && rows[w.r].ok[kKind - 1] && lm.gl < (k1 ? g.G1 : g.G2);
  return lm;
}
__device__ __forceinline__ LaneMap lane_map(const Geo& g, const Work& w, int lane, const RowPtr* rows) {
  return w.kind == 1 ? lane_map_k<1>(g, w, lane, rows) : lane_map_k<2>(g, w, lane, rows);
}

// One lane's share of an item, held in registers.
struct ItemRegs {
  uint4 w[8];    // word rows 8*gl .. 8*gl+7, columns col .. col+3
  uint2 s;       // the 4 scales
  uint32_t z;    // zero-point byte of the 4 columns
};

__device__ __forceinline__ uint4 ldg_stream16(const void* ptr) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(ptr));
  return v;
}
__device__ __forceinline__ uint2 ldg_stream8(const void* ptr) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "l"(ptr));
  return v;
}
__device__ __forceinline__ uint32_t ldg_stream1(const void* ptr) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.u8 %0, [%1];\n" : "=h"(v) : "l"(ptr));
  return v;
}

// Issue the loads of this lane's share of item w (nothing for list entries past the end, rows of a
// non-resident expert or groups past K).
__device__ __forceinline__ void load_item(const FusedParams& p, const Work& w, int lane, const RowPtr* rows,
                                          ItemRegs& it) {
  const Geo& g = p.geo;
  const LaneMap lm = lane_map(g, w, lane, rows);
  if (!lm.valid) return;
  const int mi = w.kind - 1;
  const RowPtr& rp = rows[w.r];
  const int64_t N = w.kind == 1 ? 2 * g.I : g.H;
  const uint32_t* wp = rp.w[mi] + (int64_t)(8 * lm.gl) * N + lm.col;
#pragma unroll
  for (int k = 0; k < 8; ++k) it.w[k] = ldg_stream16(wp + (int64_t)k * N);
  it.s = ldg_stream8(rp.s[mi] + ((int64_t)lm.gl * N + lm.col) * 2);
  it.z = rp.z[mi] != nullptr ? ldg_stream1(rp.z[mi] + (int64_t)lm.gl * (N / 4) + lm.col / 4) : 0u;
}

__device__ __forceinline__ void scales4(uint2 sr, bool sbf, float (&s)[4]) {
  if (sbf) {
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&sr.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&sr.y);
    s[0] = __low2float(a); s[1] = __high2float(a); s[2] = __low2float(b); s[3] = __high2float(b);
  } else {
    const __half2 a = *reinterpret_cast<const __half2*>(&sr.x);
    const __half2 b = *reinterpret_cast<const __half2*>(&sr.y);
    s[0] = __low2float(a); s[1] = __high2float(a); s[2] = __low2float(b); s[3] = __high2float(b);
  }
}

// 4 columns x 1 group of K (8 word rows) against an activation table with kPer exponents per group
// (1: the gate_up tables, 4: the down tables, one per 32 values). wd(k) gives word row k of the 4
// columns; z = zero-point byte of the 4 columns (has_z), s = their scales. Per exponent span:
// T = 64 * sum (q - zp) x_fixed exactly, then v += T * 2^(e - 6); v * s at the end.
template <int kPer, typename WordRow>
__device__ __forceinline__ void dot_group(WordRow wd, const XTable& tb, int gl, const float (&s)[4], bool has_z,
                                          uint32_t z, float (&v)[4]) {
  constexpr int kRows = 8 / kPer;
  float f[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int sp = 0; sp < kPer; ++sp) {
    int acc[4][4];
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[c][j] = 0;
#pragma unroll
    for (int kk = 0; kk < kRows; ++kk) {
      const int k = sp * kRows + kk;
      const uint4 w = wd(k);
      const uint4* xp = reinterpret_cast<const uint4*>(tb.pairs + (gl * 8 + k) * kXRegs);
      const uint4 xa = xp[0], xb = xp[1];
      const uint32_t xr[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
      word_dot(w.x, xr, acc[0]);
      word_dot(w.y, xr, acc[1]);
      word_dot(w.z, xr, acc[2]);
      word_dot(w.w, xr, acc[3]);
    }
    const int m64x = tb.m64x[gl * kPer + sp];
    const float scl = tb.scl[gl * kPer + sp];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int zp = has_z ? (int)((z >> (2 * c)) & 3u) : 2;
      f[c] += (float)(combine_classes(acc[c]) + zp * m64x) * scl;
    }
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) v[c] = f[c] * s[c];
}

// 4 columns x 1 group of this lane from its registers against an activation table.
template <int kPer>
__device__ __forceinline__ void dot_regs(const ItemRegs& it, const XTable& tb, int gl, bool sbf, bool has_z,
                                         float (&v)[4]) {
  float s[4];
  scales4(it.s, sbf, s);
  dot_group<kPer>([&](int k) { return it.w[k]; }, tb, gl, s, has_z, it.z, v);
}

// ----------------------------------------------------------------------------- copy-engine mode
__device__ __forceinline__ uint32_t smem_u32(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 10000;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase of the given parity: try_wait suspends the thread in hardware until the
// phase completes or a system time limit passes, so a waiter costs the copy engine no polling traffic.
// Exactly one thread should wait; the others meet it at a warp or CTA barrier. Error bit 1 when the
// phase never completes.
__device__ __forceinline__ void mbar_wait(uint32_t bar, unsigned parity, unsigned* err) {
  unsigned it = 0;
  while (!mbar_try(bar, parity)) {                           // each try suspends for at most ~10 us
    if (++it > kWaitLimit) {
      flag_error(err, 2u);
      return;
    }
  }
}
// L2 policy of the weight stream: evict first. Every expert byte is read once per layer, so the weights should
// not push the routing, activations and workspace words of the next layers out of L2 (0 to 0.1 us per
// config-1 layer in three A/B runs: a small effect, kept because the weights are never re-read soon).
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
      "{%2, %3, %4}], [%5], %6;\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
      "{%2, %3, %4, %5}], [%6], %7;\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void st_volatile_shared(int* ptr, int v) {
  asm volatile("st.volatile.shared.s32 [%0], %1;\n" ::"r"(smem_u32(ptr)), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_volatile_shared(const int* ptr) {
  int v;
  asm volatile("ld.volatile.shared.s32 %0, [%1];\n" : "=r"(v) : "r"(smem_u32(ptr)) : "memory");
  return v;
}
// Bounded wait until the producer has armed stage `st` for item `seq` (error bit 1 when it never does).
__device__ __forceinline__ void wait_tag(const int* tags, int st, int seq, unsigned* err) {
  unsigned it = 0;
  while (ld_volatile_shared(tags + st) != seq) {
    if (++it > kSpinLimit) {
      flag_error(err, 2u);
      return;
    }
  }
}

// Item i of the CTA's order: its phase-1 range first, then (unit, item within unit) of phase 2.
__device__ __forceinline__ Work cta_item(const Geo& g, const LiveRows& lv, const WarpList& L, int cta, int i) {
  Work w{};
  if (i < L.range) {
    const int ii = L.a + i;
    const int per_row = g.nb1 * g.kp1;
    w.kind = 1;
    const int rc = fdiv(ii, g.d_row1);
    w.r = lv.rowmap[rc];
    const int rem = ii - rc * per_row;
    w.b = fdiv(rem, g.d_kp1);
    w.kp = rem - w.b * g.kp1;
    return w;
  }
  const int i2 = i - L.range;
  const int q = fdiv(i2, g.d_s2), j = i2 - q * g.s2;
  const int u = cta + g.grid * q, m = fdiv(u, g.d_nb2);
  w.kind = 2;
  w.b = u - m * g.nb2;
  unit_row(g, lv, m, j, w);
  return w;
}

// Copy descriptor of item i of the CTA's order: {kind (0 = nothing to copy), slot, block, K-part};
// slot_of(r, kind) = arena slot of routed row r's expert for that projection, -1 when it does not resolve.
template <class SlotOf>
__device__ __forceinline__ int4 item_desc(const Geo& g, const LiveRows& lv, const WarpList& L0, int cta,
                                          SlotOf slot_of, int i) {
  const Work w = cta_item(g, lv, L0, cta, i);
  const int sl = w.dead ? -1 : slot_of(w.r, w.kind);
  const bool live = sl >= 0;                                  // slot_of returns -1 for slots >= S
  return make_int4(live ? w.kind : 0, sl, w.b, w.kp);
}

// The producers: issuing thread k (lane k / kProducers of producer warp k % kProducers) streams items
// k, k + kIssuers, ... of the CTA's order through the ring. One issuing thread sustains only about an
// eighth of an SM's share of HBM bandwidth (each arm-and-copy sequence has a long latency), so several
// issue side by side; two lanes of one warp issue in the same instructions. The warp's lanes decode its
// next 32 descriptors in parallel. The stage count is a multiple of kIssuers, so every stage has a single
// issuer. Each item is one tensor copy of codes (4 KB), one of scales and one of zero-point windows,
// completing on the stage's `full` barrier; a stage is refilled once the warp that reduced it arrived on
// its `empty` barrier. Items of a non-resident expert complete their phase on the arrival alone.
template <class SlotOf>
__device__ void produce(const FusedParams& p, const LiveRows& lv, SlotOf slot_of, int cta, unsigned char* stages,
                        uint32_t bars, int* tags, int pr, int lane) {
  const Geo& g = p.geo;
  const WarpList L0 = warp_list(g, lv, cta, 0);
  const int n = L0.range + L0.nu * g.s2;
  const int nw = n > pr ? (n - pr + kProducers - 1) / kProducers : 0;   // items of this warp: pr + kProducers*j
  const int ns = p.nstage;
  const bool hz = p.map13.has_zeros != 0;
  const bool aligned = (smem_u32(stages) & 127u) == 0;        // tensor copies land on 128-byte boundaries
  if (!aligned && lane == 0) flag_error(p.err, 4u);
  const bool issuer = lane < kIssuers / kProducers;
  const uint64_t pol = evict_first_policy();
  int4 batch = make_int4(0, 0, 0, 0);
  for (int j0 = 0; j0 < nw; j0 += kIssuers / kProducers) {
    if ((j0 & 31) == 0) {
      const int ii = pr + kProducers * (j0 + lane);
      batch = j0 + lane < nw ? item_desc(g, lv, L0, cta, slot_of, ii) : make_int4(0, 0, 0, 0);
    }
    const int src = (j0 & 31) + (lane & 1);
    int4 it;
    it.x = __shfl_sync(0xffffffffu, batch.x, src);
    it.y = __shfl_sync(0xffffffffu, batch.y, src);
    it.z = __shfl_sync(0xffffffffu, batch.z, src);
    it.w = __shfl_sync(0xffffffffu, batch.w, src);
    const int j = j0 + lane;
    if (issuer && j < nw) {
      const int i = pr + kProducers * j;
      const int st = i % ns, round = i / ns;
      const uint32_t full = bars + st * 8, empty = bars + (ns + st) * 8;
      if (round > 0) mbar_wait(empty, (unsigned)(round - 1) & 1u, p.err);
      // Tag the stage with the item it now holds. A warp waits for its item's tag before it waits on the
      // stage's `full` phase: a stage is refilled by another warp's item, and without the tag a warp that
      // runs ahead could take the still-pending previous fill's phase parity for its own.
      st_volatile_shared(tags + st, i);
      if (!aligned || it.x == 0) {
        mbar_arrive(full);
      } else {
        const uint32_t dst = smem_u32(stages + (size_t)st * kStageBytes);
        mbar_arrive_tx(full, (unsigned)(kScaleOff + 256 + (hz ? 64 : 0)));
        const int zx = (8 * it.z) & ~15;                      // 16-byte aligned zero-point window
        if (it.x == 1) {
          tma_load_4d(dst, &p.tm[0], it.z * 32, 0, 16 * it.w, it.y, full, pol);
          tma_load_4d(dst + kScaleOff, &p.tm[1], it.z * 32, 0, 2 * it.w, it.y, full, pol);
          if (hz) tma_load_4d(dst + kZeroOff, &p.tm[2], zx, 0, 2 * it.w, it.y, full, pol);
        } else {
          tma_load_3d(dst, &p.tm[3], it.z * 32, 32 * it.w, it.y, full, pol);
          tma_load_3d(dst + kScaleOff, &p.tm[4], it.z * 32, 4 * it.w, it.y, full, pol);
          if (hz) tma_load_3d(dst + kZeroOff, &p.tm[5], zx, 4 * it.w, it.y, full, pol);
        }
      }
    }
    __syncwarp();
  }
  // every copy has landed before the producer leaves (the reducing warps wait on the same phases)
  if (issuer)
    for (int s0 = pr + kProducers * lane; s0 < ns && s0 < n; s0 += kIssuers) {
      const int last = s0 + ((n - 1 - s0) / ns) * ns;
      mbar_wait(bars + s0 * 8, (unsigned)(last / ns) & 1u, p.err);
    }
}

// 4 columns x 1 group of this lane from a ring stage. Gate_up stages hold 256-byte word rows (32 gate |
// 32 up columns), scales [group][half][32] and zero windows [group][half][16 B]; down stages 128-byte
// rows, scales [group][32] and windows [group][16 B].
template <int kPer, int kKind>
__device__ __forceinline__ void dot_stage(const unsigned char* st, const Work& w, int lane, const XTable& tb, int gl,
                                          bool sbf, bool has_z, float (&v)[4]) {
  constexpr bool k1 = kKind == 1;
  const int gi = k1 ? (lane >> 4) : (lane >> 3);
  const int q = k1 ? (lane & 15) : (lane & 7);
  const int side = k1 && q >= 8 ? 1 : 0;
  const int q8 = k1 ? (q & 7) : q;
  const int row_bytes = k1 ? 256 : 128;
  const int sub = k1 ? gi * 2 + side : gi;                   // (group, half) index of scales / windows
  const unsigned char* code = st + (size_t)(8 * gi) * row_bytes + side * 128 + q8 * 16;
  const uint2 sr = *reinterpret_cast<const uint2*>(st + kScaleOff + (sub * 32 + q8 * 4) * 2);
  float s[4];
  scales4(sr, sbf, s);
  const uint32_t zbyte = has_z ? (uint32_t)st[kZeroOff + sub * 16 + ((8 * w.b) & 15) + q8] : 0u;
  dot_group<kPer>([&](int k) { return *reinterpret_cast<const uint4*>(code + k * row_bytes); }, tb, gl, s, has_z,
                  zbyte, v);
}


// One item of kind kKind (1 gate_up, 2 down; compile-time, so each loop carries only its own inner product).
template <bool kTma, int kKind>
__device__ __forceinline__ void process_work(const FusedParams& p, const Work& w, int lane, const ItemRegs& it,
                                             const unsigned char* stage, unsigned char* smem, float* mail1,
                                             float* mail2, const RowPtr* rows) {
  const Geo& g = p.geo;
  constexpr bool k1 = kKind == 1;
  constexpr int mi = kKind - 1;
  const RowPtr& rp = rows[w.r];
  unsigned char* tabs = smem + p.off_tabs;
  const LaneMap lm = lane_map_k<kKind>(g, w, lane, rows);
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  if (lm.valid) {
    const bool sbf = p.scale_bf16 != 0, hz = rp.z[mi] != nullptr;
    if constexpr (k1) {
      const XTable tb = table_at(tabs + (size_t)fdiv(w.r, g.d_topk) * token_table_bytes(g.H), g.H);
      if constexpr (kTma) dot_stage<1, 1>(stage, w, lane, tb, lm.gl, sbf, hz, v);
      else dot_regs<1>(it, tb, lm.gl, sbf, hz, v);
    } else {
      const XTable tb = htable_at(tabs + (size_t)w.jr * htab_bytes(g.I), g.I);
      if constexpr (kTma) dot_stage<kGroup / kSub, 2>(stage, w, lane, tb, lm.gl, sbf, hz, v);
      else dot_regs<kGroup / kSub>(it, tb, lm.gl, sbf, hz, v);
    }
  }
  if constexpr (k1) {
#pragma unroll
    for (int c = 0; c < 4; ++c) v[c] += __shfl_xor_sync(0xffffffffu, v[c], 16);
    if (lane < 16)
      *reinterpret_cast<float4*>(mail1 + (size_t)w.slot * 64 + lane * 4) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      v[c] += __shfl_xor_sync(0xffffffffu, v[c], 8);
      v[c] += __shfl_xor_sync(0xffffffffu, v[c], 16);
    }
    const float wr = rows[w.r].wt;
    if (lane < 8)
      *reinterpret_cast<float4*>(mail2 + (size_t)w.slot * 32 + lane * 4) =
          make_float4(v[0] * wr, v[1] * wr, v[2] * wr, v[3] * wr);
  }
}

__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* ptr) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* ptr) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_u32(unsigned* ptr, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;\n" ::"l"(ptr), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* ptr, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;\n" ::"l"(ptr), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* ptr) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];\n" : "=l"(v) : "l"(ptr) : "memory");
  return v;
}

// All CTAs arrive; thread 0 of each CTA calls this with `base`, the generation word it read at kernel
// entry. The arrival count only grows, and the generation word holds the count every completed call
// reached, so an arrival is one fire-and-forget release add and every CTA waits until the count reaches
// base + ncta (signed distance, so the words may wrap). CTA 0 then stores that value as the new
// generation, which the next call reads at entry; no CTA of this call reads it after its own entry, and
// the grid size may differ from call to call. The count sits 128 bytes away from the generation. Gives
// up after kSpinLimit polls (error bit 1). The caller brackets it with CTA barriers: the release add then
// publishes every write the CTA made before the first one, and the acquire load orders every read the
// CTA makes after the second one (no full fences, which stall for microseconds under the weight stream).
__device__ void grid_barrier(unsigned* count, unsigned* gen, unsigned base, unsigned ncta, unsigned* err) {
  asm volatile("red.release.gpu.global.add.u32 [%0], 1;\n" ::"l"(count) : "memory");
  const unsigned target = base + ncta;
  unsigned it = 0;
  while ((int)(ld_acquire_u32(count) - target) < 0) {
    if (++it > kSpinLimit) {
      flag_error(err, 2u);
      break;
    }
  }
  if (blockIdx.x == 0) st_release_u32(gen, target);
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, unsigned bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// Items [0, head_k) of a CTA's range are the tail of an h-block that began in the previous CTA. Once
// they are reduced (round 0 of the item loop), the warp that completes them sums their partials and
// publishes the (gate, up) tail sums of its 32 columns, so the previous CTA can finish that block before
// the grid barrier. Each sum travels with the call's epoch in one 64-bit word (single-copy atomic), so
// the reader needs no flag and neither side a fence -- a release store here would stall the warp until
// its earlier stores drain, for microseconds under the weight stream.
__device__ void publish_head(const FusedParams& p, int cta, int lane, const float* mail1, int head_k,
                             unsigned epoch) {
  __syncwarp();                                               // the warps' partials are in place (counter)
  float gs = 0.f, us = 0.f;
  for (int i = 0; i < head_k; ++i) {
    gs += mail1[(size_t)i * 64 + lane];
    us += mail1[(size_t)i * 64 + 32 + lane];
  }
  const unsigned long long tag = (unsigned long long)epoch << 32;
  unsigned long long* slot = p.hand + (size_t)cta * 64;
  st_relaxed_u64(slot + lane, tag | __float_as_uint(gs));
  st_relaxed_u64(slot + 32 + lane, tag | __float_as_uint(us));
}

// Count one reduced head item; the warp that reduces the last of them publishes the tail sums.
__device__ __forceinline__ void head_item_done(const FusedParams& p, const LiveRows& lv, const WarpList& L, int cta,
                                               int lane, const float* mail1, int head_k, unsigned epoch,
                                               unsigned* counter) {
  unsigned last = 0u;
  if (lane == 0) {
    __threadfence_block();
    last = atomicAdd(counter, 1u) == (unsigned)head_k - 1u;
    __threadfence_block();
  }
  if (__shfl_sync(0xffffffffu, last, 0)) publish_head(p, cta, lane, mail1, head_k, epoch);
}

// Phase switch, entered by every warp of the CTA once its gate_up items are done. (1) h of every h-block
// this CTA finishes, in item order, into the down tables: whole blocks from its own partials; the block it
// shares with the next CTA from its head part plus the tail sums that CTA published (bounded wait on its
// flag); the block it shares with the previous CTA is finished there. (2) Grid barrier: the tables are
// complete.
__device__ __forceinline__ void phase_switch(const FusedParams& p, const LiveRows& lv, int cta, int warp, int lane,
                                             const float* mail1, unsigned epoch) {
  const Geo& g = p.geo;
  const WarpList L = warp_list(g, lv, cta, warp);
  csync();
  {
    const long long a = L.a, b = L.b;
    if (b > a) {
      const int blk0 = fdiv((int)a, g.d_kp1), blk1 = fdiv((int)(b - 1), g.d_kp1);
      for (int blk = blk0 + warp; blk <= blk1; blk += kWarps) {
        const long long i0 = (long long)blk * g.kp1, i1 = i0 + g.kp1;
        if (i0 < a) continue;                                 // finished by the previous CTA
        const long long hi = i1 < b ? i1 : b;
        float gs = 0.f, us = 0.f;
        for (long long i = i0; i < hi; ++i) {
          gs += mail1[(size_t)(i - a) * 64 + lane];
          us += mail1[(size_t)(i - a) * 64 + 32 + lane];
        }
        const int rc = fdiv(blk, g.d_nb1), hb = blk - rc * g.nb1;
        const int r = lv.rowmap[rc];
        if (i1 > b) {                                         // tail published by the next CTA (bounded wait)
          const unsigned long long* slot = p.hand + (size_t)(cta + 1) * 64;
          unsigned long long vg = 0, vu = 0;
          unsigned it = 0;
          while (true) {
            vg = ld_relaxed_u64(slot + lane);
            vu = ld_relaxed_u64(slot + 32 + lane);
            if ((unsigned)(vg >> 32) == epoch && (unsigned)(vu >> 32) == epoch) break;
            if (++it > kSpinLimit) {
              flag_error(p.err, 2u);
              break;
            }
            __nanosleep(32);
          }
          __syncwarp();
          gs += __uint_as_float((unsigned)vg);
          us += __uint_as_float((unsigned)vu);
        }
        htab_block(p.htab + (size_t)r * htab_bytes(g.I), g.I, hb, silu(gs) * us, lane);
      }
    }
  }
  csync();
  if (threadIdx.x == 0) grid_barrier(p.bar_count, p.bar_gen, epoch - 1u, gridDim.x, p.err);
  csync();
  // Every CTA of this grid is resident: the next kernel of the stream may be scheduled as SMs free up (its
  // CTAs wait for this grid's completion before reading anything it writes).
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

}

// The down unit q of this CTA (token m, 32 output columns): the h tables of its live routed rows ->
// shared memory (table slot jr), one bulk copy each. Starts with a barrier of the reducing warps (the
// previous unit's tables are free; the phase switch ends with one before unit 0) and ends with one (this
// unit's are in place). The live rows of a unit are its token's first tokcnt[m] table slots.
__device__ __forceinline__ void unit_tables(const FusedParams& p, const LiveRows& lv, int cta, int q,
                                            unsigned char* smem, uint32_t hbar) {
  const Geo& g = p.geo;
  const int* slotrow = lv.slotrow + q * g.top_k;
  const size_t tb = htab_bytes(g.I);
  if (q > 0) csync();
  if (threadIdx.x == 0) {
    const int u = cta + g.grid * q;
    const unsigned live = u < g.u2 ? (unsigned)lv.tokcnt[fdiv(u, g.d_nb2)] : 0u;
    mbar_arrive_tx(hbar, (unsigned)tb * live);
  }
  if (threadIdx.x < g.top_k && slotrow[threadIdx.x] >= 0) {
    asm volatile("fence.proxy.async.global;\n" ::: "memory");  // the tables were written through the generic proxy
    bulk_g2s(smem_u32(smem + p.off_tabs + (size_t)threadIdx.x * tb), p.htab + (size_t)slotrow[threadIdx.x] * tb,
             (unsigned)tb, hbar);
  }
  if (threadIdx.x == 0) mbar_wait(hbar, (unsigned)q & 1u, p.err);
  csync();
}

// kTma = false: register mode (any expert map), 512 threads; every lane loads its item data itself.
// kTma = true: copy-engine mode (slot arenas), 512 reducing threads + one producer warp.
// kEx: the expert-parallel exchange variant (p.xin / p.yout honoured); the plain variant carries none of it.
template <bool kTma, bool kEx>
__global__ void __launch_bounds__(kTma ? kTmaThreads : kThreads, 1) fused_layer_kernel(const __grid_constant__ FusedParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const Geo& g = p.geo;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  float* mail1 = reinterpret_cast<float*>(smem + p.off_mail1);
  float* mail2 = reinterpret_cast<float*>(smem + p.off_mail2);
  RowPtr* rows = reinterpret_cast<RowPtr*>(smem + p.off_rows);
  unsigned* misc = reinterpret_cast<unsigned*>(smem + p.off_misc);  // [0,1] h-copy mbarrier, [2] head count,
                                                                    // [3] grid barrier generation at entry
  const uint32_t hbar = smem_u32(misc);
  unsigned char* stages = kTma ? smem + p.off_stages : nullptr;
  const uint32_t bars = kTma ? smem_u32(smem + p.off_bars) : 0u;
  int* tags = kTma ? reinterpret_cast<int*>(smem + p.off_bars + 16 * (size_t)p.nstage) : nullptr;

  if (kTma && warp >= kWarps) {
    // producer warps: ring barriers and stage tags, and the tensor maps into the descriptor cache
    const int pt = threadIdx.x - kThreads;
    for (int b = pt; b < 2 * p.nstage; b += 32 * kProducers) {
      mbar_init(bars + b * 8, 1);                             // full[0..ns), then empty[0..ns)
      if (b < p.nstage) tags[b] = -1;
    }
    if (pt == 0) mbar_init(hbar, 1);                          // the h-table copies' barrier
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    if (pt < 6 && (p.map13.has_zeros || (pt != 2 && pt != 5)))
      asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&p.tm[pt])) : "memory");
  }
  // The slot table, staged into shared memory while the previous kernel may still be finishing: the kernels
  // that let this one start early (this library's layer, INT8 and all-reduce kernels, which trigger their
  // dependents before they end) never write a slot table, and any other kernel -- or a copy -- that writes
  // one has completed before this kernel starts.
  const bool one_warp = g.R <= 32;
  int* sltab = reinterpret_cast<int*>(smem + p.off_slots);    // staged slot table (g.stab entries)
  if (one_warp && g.stab > 0) {
    if (warp == 0) stage_slots(sltab, p.map13.slots, g.stab, lane);
    if (kTma && warp >= kWarps && private_routing(g))
      stage_slots(reinterpret_cast<int*>(smem + p.off_preg) + (warp - kWarps) * preg_ints(g) + 128, p.map13.slots,
                  g.stab, lane);
  }
  // Launched with programmatic stream serialisation, this CTA may start while the previous kernel of the
  // stream is finishing: everything above touches only shared memory, the kernel's own parameters and the
  // slot table; from here on it reads what earlier work wrote (routing, activations, workspace, weights).
  asm volatile("griddepcontrol.wait;\n" ::: "memory");

  // the barrier generation of this call (read at entry; the count reaches it before any CTA of this call
  // can pass the barrier). The previous call stored it before it ended, so stream order alone makes it
  // visible: a relaxed load, which -- unlike an acquire -- does not hold back this thread's routing loads.
  const unsigned gen_entry = threadIdx.x == 0 ? ld_relaxed_u32(p.bar_gen) : 0u;
  // expert parallelism: the call this layer pushes, read before any CTA can pass the grid barrier (CTA 0 advances
  // the channel after it)
  const unsigned e_out = kEx && p.yout && warp == 0 ? ld_relaxed_gpu_u32(p.xepoch) + 1u : 0u;
  int* rowmap = reinterpret_cast<int*>(smem + p.off_live);
  int* tokrow = rowmap + g.R;
  int* tokcnt = tokrow + g.R;
  int* slotrow = tokcnt + g.M;
  unsigned* livebits = reinterpret_cast<unsigned*>(slotrow + g.max_units * g.top_k);
  // Routing first: expert bases of every routed row, resolved once per CTA -- by warp 0 alone when the
  // rows fit one warp (it compacts them right after, with no CTA barrier in between), else by every thread.
  auto resolve_row = [&](int r, int e, float wt, bool staged) {
    RowPtr rp;
    rp.wt = wt;
    if (staged) {                                             // one shared slot table for both projections
      const bool in = e >= 0 && e < p.map13.E;
      if (!in) flag_error(p.err, 1u);
      const int sl = in ? sltab[e] : -1;
      rp.ok[0] = in && p.map13.resolve_slot(sl, rp.w[0], rp.s[0], rp.z[0], p.err);
      rp.ok[1] = in && p.map2.resolve_slot(sl, rp.w[1], rp.s[1], rp.z[1], nullptr);
      rp.slot = sl < p.map13.S ? sl : -1;
    } else {
      rp.ok[0] = p.map13.resolve(e, rp.w[0], rp.s[0], rp.z[0], p.err);
      rp.ok[1] = p.map2.resolve(e, rp.w[1], rp.s[1], rp.z[1], p.err);
      rp.slot = (p.map13.slots != nullptr && e >= 0 && e < p.map13.E) ? p.map13.slots[e] : -1;
      if (rp.slot >= p.map13.S) rp.slot = -1;                 // (resolve flagged it)
    }
    rows[r] = rp;
  };
  if (one_warp) {
    // warp 0: the routing in one round of loads, then lookups in the staged slot table
    if (warp == 0) {
      const int e = lane < g.R ? p.ids[lane] : -1;
      const float wt = lane < g.R ? p.topk_w[lane] : 0.f;
      __syncwarp();
      if (lane < g.R) resolve_row(lane, e, wt, g.stab > 0);
    }
  } else {
    for (int r = threadIdx.x; r < g.R; r += blockDim.x) resolve_row(r, p.ids[r], p.topk_w[r], false);
  }
  if (!kTma) {
    // Start the whole layer's weight stream: this CTA's 1/grid share of every routed row's six arrays.
    // A prefetch is only a hint, so arrays whose base is not 16-byte aligned are left to the loads.
    for (int idx = threadIdx.x; idx < g.R * 6; idx += blockDim.x) {
      const int r = idx / 6, arr = idx - r * 6, ph = arr / 3, kind = arr - ph * 3;
      const ExpertMap& mp = ph == 0 ? p.map13 : p.map2;
      const uint32_t* wb = nullptr;
      const char* sb = nullptr;
      const uint8_t* zb = nullptr;
      if (!mp.resolve(p.ids[r], wb, sb, zb, nullptr)) continue;
      const int64_t K = ph == 0 ? g.H : g.I, N = ph == 0 ? 2 * g.I : g.H;
      const char* base = kind == 0 ? reinterpret_cast<const char*>(wb)
                                   : (kind == 1 ? sb : reinterpret_cast<const char*>(zb));
      const int64_t bytes =
          kind == 0 ? (K / 16) * N * 4 : (kind == 1 ? (K / kGroup) * N * 2 : (K / kGroup) * (N / 4));
      if (base == nullptr || (reinterpret_cast<uintptr_t>(base) & 15u)) continue;
      const int64_t chunk = ((bytes + g.grid - 1) / g.grid + 15) & ~int64_t(15);
      const int64_t start = (int64_t)cta * chunk;
      const int64_t len = (start < bytes ? (bytes - start < chunk ? bytes - start : chunk) : 0) & ~int64_t(15);
      if (len > 0)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(base + start), "r"((unsigned)len) : "memory");
    }
  }

  // activation tables of the M rows of x (no dependence on the routing), by reducing warps 1..15
  if (warp >= 1 && warp < kWarps) {
    // expert parallelism: x = the ranks' rows of the channel's call e, once every rank's flag has reached e
    // expert parallelism: x = the ranks' tagged rows of the channel's call e, each word used once it holds e
    const unsigned long long* xsum = nullptr;
    unsigned e_in = 0, budget = p.xspin;
    if (kEx && p.xin) {
      e_in = ld_relaxed_gpu_u32(p.xepoch);
      xsum = reinterpret_cast<const unsigned long long*>(p.xpeers[p.xrank] + p.xtag_off) +
             (size_t)(e_in & 1u) * p.xworld * (p.xn_max / 2);
    }
    // the 4 values of x row m, group gi this lane converts
    auto load_x4 = [&](int m, int gi, float (&v)[4]) {
      const size_t off = (size_t)m * g.H + gi * kGroup + 4 * lane;
      if (!kEx || xsum == nullptr) {
        const __nv_bfloat162* src = reinterpret_cast<const __nv_bfloat162*>(p.x + off);
        const float2 a0 = __bfloat1622float2(src[0]), a1 = __bfloat1622float2(src[1]);
        v[0] = a0.x; v[1] = a0.y; v[2] = a1.x; v[3] = a1.y;
      } else {
        // the ranks' rows in rank order, summed in fp32 and rounded to bf16 as the all-reduce does
        float s[4] = {0.f, 0.f, 0.f, 0.f};
        for (int r = 0; r < p.xworld; ++r) {
          const unsigned long long* row = xsum + (size_t)r * (p.xn_max / 2) + off / 2;
          const float2 a0 = bf16x2_to_float2(wait_tagged(row, e_in, budget, p.err));
          const float2 a1 = bf16x2_to_float2(wait_tagged(row + 1, e_in, budget, p.err));
          s[0] += a0.x; s[1] += a0.y; s[2] += a1.x; s[3] += a1.y;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __bfloat162float(__float2bfloat16(s[i]));
      }
    };
    constexpr int kXW = kWarps - 1, kXPre = 4;
    const int xw = warp - 1, nxt = g.M * g.G1;
    float xv[kXPre][4];
    int gl[kXPre], toff[kXPre];
#pragma unroll
    for (int j = 0; j < kXPre; ++j) {
      const int t = xw + j * kXW;
      const int m = fdiv(t, g.d_G1), gi = t - m * g.G1;
      xv[j][0] = xv[j][1] = xv[j][2] = xv[j][3] = 0.f;
      gl[j] = -1;
      toff[j] = 0;
      if (t < nxt) {
        load_x4(m, gi, xv[j]);
        gl[j] = gi;
        toff[j] = m * (int)token_table_bytes(g.H);
      }
    }
    prep_groups<kXPre>(xv, gl, toff, smem + p.off_tabs, g.H, lane);
    for (int tt = xw + kXPre * kXW; tt < nxt; tt += kXW) {
      const int m = fdiv(tt, g.d_G1), gi = tt - m * g.G1;
      float v[4];
      load_x4(m, gi, v);
      prep_group_regs(v, gi, table_at(smem + p.off_tabs + (size_t)m * token_table_bytes(g.H), g.H), lane);
    }
  }
  if (!one_warp) __syncthreads();
  // Live routed rows (both experts resolve), compacted by warp 0 with ballots: rowmap in routing order,
  // and per token its live rows' positions within its top_k. The producers start as soon as warp 0 is
  // done (they need the routing, not the activation tables).
  if (warp == 0) {
    __syncwarp();
    int nl = 0;
    for (int c0 = 0; c0 < g.R; c0 += 32) {
      const int r = c0 + lane;
      const bool live = r < g.R && rows[r].ok[0] && rows[r].ok[1];
      const unsigned bal = __ballot_sync(0xffffffffu, live);
      if (live) rowmap[nl + __popc(bal & ((1u << lane) - 1u))] = r;
      if (lane == 0) livebits[c0 >> 5] = bal;
      nl += __popc(bal);
    }
    __syncwarp();
    for (int m = lane; m < g.M; m += 32) {
      int c = 0;
      for (int j = 0; j < g.top_k; ++j) {
        const int r = m * g.top_k + j;
        if ((livebits[r >> 5] >> (r & 31)) & 1u) tokrow[m * g.top_k + c++] = j;
      }
      tokcnt[m] = c;
    }
    if (lane == 0) {
      if (!kTma) {                                            // (copy-engine mode: the producers set it up)
        mbar_init(hbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
      }
      misc[2] = 0u;
      misc[3] = gen_entry;                 // read by every CTA before any passes this call's barrier
      const int nblk = nl * g.nb1;
      misc[4] = (unsigned)(nblk * g.kp1);
      misc[5] = (unsigned)max(1, min((int)gridDim.x, nblk));
    }
    if (kTma && !private_routing(g)) bar_arrive(2, 32 * (kProducers + 1));
  }
  if constexpr (kTma) {
   if (warp >= kWarps) {
    bar_arrive(3, kTmaThreads);                               // ring barriers and tags initialised
    const int pw = warp - kWarps;
    if (private_routing(g)) {
      // This warp's own copy of the routing, by the rules warp 0 applies for the reducing warps (the same
      // live rows in the same order): the ids in one round of loads, lookups in its staged slot table,
      // ballot compaction.
      int* reg = reinterpret_cast<int*>(smem + p.off_preg) + pw * preg_ints(g);
      int* pslot = reg;
      int* prow = reg + 32;
      int* ptokrow = reg + 64;
      int* ptokcnt = reg + 96;
      int* pstab = reg + 128;
      const int e = lane < g.R ? p.ids[lane] : -1;      // (the slot table was staged before the wait)
      __syncwarp();
      const bool in = lane < g.R && e >= 0 && e < p.map13.E;
      const int sl = in ? pstab[e] : -1;
      const bool live = in && sl >= 0 && sl < p.map13.S;      // the rule resolve_slot applies
      const unsigned bal = __ballot_sync(0xffffffffu, live);
      pslot[lane] = live ? sl : -1;
      if (live) prow[__popc(bal & ((1u << lane) - 1u))] = lane;
      if (lane < g.M) {
        unsigned bits = (bal >> (lane * g.top_k)) & (g.top_k >= 32 ? 0xffffffffu : (1u << g.top_k) - 1u);
        int c = 0;
        while (bits) {
          ptokrow[lane * g.top_k + c++] = __ffs(bits) - 1;
          bits &= bits - 1u;
        }
        ptokcnt[lane] = c;
      }
      __syncwarp();
      const int nblk = __popc(bal) * g.nb1;
      const LiveRows plv{prow, ptokrow, ptokcnt, nullptr, nblk * g.kp1, max(1, min((int)gridDim.x, nblk))};
      produce(p, plv, [&](int r, int) { return pslot[r]; }, cta, stages, bars, tags, pw, lane);
    } else {
      bar_wait(2, 32 * (kProducers + 1));                     // routing compacted by warp 0
      const LiveRows lv{rowmap, tokrow, tokcnt, slotrow, (int)misc[4], (int)misc[5]};
      produce(p, lv, [&](int r, int kind) { const RowPtr& rp = rows[r]; return rp.ok[kind - 1] ? rp.slot : -1; }, cta,
              stages, bars, tags, pw, lane);
    }
    return;
   }
  }
  if (kTma) bar_wait(3, kTmaThreads);                         // reducing warps: tables, routing, ring ready
  else csync();
  const LiveRows lv{rowmap, tokrow, tokcnt, slotrow, (int)misc[4], (int)misc[5]};
  const WarpList L = warp_list(g, lv, cta, warp);
  for (int idx = threadIdx.x; idx < g.max_units * g.top_k; idx += kThreads) {   // rows of the CTA's down units
    const int q = fdiv(idx, g.d_topk), jr = idx - q * g.top_k, u = cta + g.grid * q;
    int row = -1;
    if (u < g.u2) {
      const int m = fdiv(u, g.d_nb2);
      if (jr < tokcnt[m]) row = m * g.top_k + tokrow[m * g.top_k + jr];
    }
    slotrow[idx] = row;                    // read after the phase switch's barriers
  }

  // The warp's work list: its gate_up items, the phase switch, then unit by unit its down items (each unit
  // preceded by the unit's h tables and followed by the unit's y). Register mode: take the item whose loads
  // are in flight, issue the next one's, reduce. Copy-engine mode: wait for the item's ring stage, reduce,
  // release the stage.
  const unsigned epoch = misc[3] + 1u;
  const int head_k = L.a % g.kp1 ? min(g.kp1 - L.a % g.kp1, L.range) : 0;   // items finishing a shared block
  const int total = L.total();
  auto item_at = [&](int t) -> Work {                         // register mode look-ahead only
    if (t < L.n1w) return work1(g, lv, L, warp, t);
    const int t2 = t - L.n1w;
    if (L.n2w == 0 || t2 >= L.nu * L.n2w) return Work{};
    const int q = t2 / L.n2w;
    return work2(g, lv, L, cta, warp, q, t2 - q * L.n2w);
  };
  ItemRegs cur, nxt_it;
  Work wn{};
  if (!kTma) {
    wn = item_at(0);
    load_item(p, wn, lane, rows, nxt_it);
  }
  int tr = 0;                                                 // register mode: flat index of the item
  auto do_item = [&](const Work& w, auto kind) {
    constexpr int K = decltype(kind)::value;
    if constexpr (kTma) {
      const int st = w.seq % p.nstage;
      if (lane == 0) {
        wait_tag(tags, st, w.seq, p.err);
        mbar_wait(bars + st * 8, (unsigned)(w.seq / p.nstage) & 1u, p.err);
      }
      __syncwarp();
      process_work<true, K>(p, w, lane, cur, stages + (size_t)st * kStageBytes, smem, mail1, mail2, rows);
      __syncwarp();
      if (lane == 0) mbar_arrive(bars + (p.nstage + st) * 8);
      if constexpr (K == 1)
        if (w.slot < head_k) head_item_done(p, lv, L, cta, lane, mail1, head_k, epoch, misc + 2);
    } else {
      const Work wc = wn;
      cur = nxt_it;
      if (++tr < total) {
        wn = item_at(tr);
        load_item(p, wn, lane, rows, nxt_it);
      }
      process_work<false, K>(p, wc, lane, cur, nullptr, smem, mail1, mail2, rows);
      __syncwarp();
      if constexpr (K == 1)
        if (wc.slot < head_k) head_item_done(p, lv, L, cta, lane, mail1, head_k, epoch, misc + 2);
    }
  };
  for (int t = 0; t < L.n1w; ++t) do_item(work1(g, lv, L, warp, t), std::integral_constant<int, 1>{});
  phase_switch(p, lv, cta, warp, lane, mail1, epoch);
  for (int q = 0; q < L.nu; ++q) {
    unit_tables(p, lv, cta, q, smem, hbar);
    for (int k = 0; k < L.n2w; ++k) do_item(work2(g, lv, L, cta, warp, q, k), std::integral_constant<int, 2>{});
    csync();
    if (warp == 0) {                          // y of the unit: fixed-order sum of its top_k x K-part partials
      const int u = cta + g.grid * q, m = fdiv(u, g.d_nb2), b = u - m * g.nb2;
      float acc = 0.f;
      for (int j = 0; j < g.s2; ++j) acc += mail2[(size_t)j * 32 + lane];
      const __nv_bfloat16 v = __float2bfloat16(acc * p.rsf);
      if (kEx && p.yout) {                    // this rank's tagged row of call e_out, into every rank's buffer
        const uint32_t mine = (uint32_t)__bfloat16_as_ushort(v);
        const uint32_t next = __shfl_down_sync(0xffffffffu, mine, 1);
        if ((lane & 1) == 0) {
          const unsigned long long word = ((unsigned long long)e_out << 32) | (next << 16) | mine;
          const size_t wi = ((size_t)(e_out & 1u) * p.xworld + p.xrank) * (p.xn_max / 2) +
                            ((size_t)m * g.H + b * 32 + lane) / 2;
          for (int r = 0; r < p.xworld; ++r)
            st_tagged(reinterpret_cast<unsigned long long*>(p.xpeers[r] + p.xtag_off) + wi, word);
        }
      } else {
        p.y[(int64_t)m * g.H + b * 32 + lane] = v;
      }
    }
  }
  // the next kernel reads *xepoch only after this grid has completed; no CTA reads it after the grid barrier
  if (kEx && p.yout && cta == 0 && warp == 0 && lane == 0)
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;\n" ::"l"(p.xepoch), "r"(e_out) : "memory");
}

}  // namespace

// Workspace: 256 bytes of control words (grid barrier arrival count at 0 and generation at 128; both
// only grow and are equal between calls, so zero-filling before the first call is all they need),
// kMaxGrid x 512 bytes of hand-off words (tagged with past epochs, never reset; zero qualifies), then the
// down tables of the routed rows [R][htab_bytes(I)] (2.25 I bytes each).
constexpr int kMaxGrid = 256;
constexpr size_t kHandBytes = (size_t)kMaxGrid * 64 * 8;
size_t layer_workspace_bytes(int M, int H, int I, int top_k) {
  (void)H;
  const size_t head = 256 + kHandBytes;
  if (M <= 0 || I <= 0 || top_k <= 0) return head;
  return head + (size_t)M * top_k * htab_bytes(I);
}

namespace {

// ----------------------------------------------------------------------------- host side
// Shared-memory plan of copy-engine mode: the ring first (offset 0, so every stage is 128-byte aligned),
// then the plan of register mode, then 2 * nstage mbarriers and nstage stage tags. Returns 0 stages when
// fewer than kMinStages fit.
struct TmaPlan {
  int nstage;
  size_t stages, rest, total;
};
TmaPlan tma_plan(const Geo& g) {
  TmaPlan t{};
  const size_t cap = 227 * 1024;
  t.rest = smem_plan(g).total;
  const size_t fixed = t.rest + 2 * kMaxStages * 8 + kMaxStages * 4;
  int ns = fixed < cap ? (int)((cap - fixed) / kStageBytes) : 0;
  if (ns > kMaxStages) ns = kMaxStages;
  ns -= ns % kIssuers;
  t.nstage = ns >= kMinStages ? ns : 0;
  t.stages = (size_t)t.nstage * kStageBytes;
  t.total = t.stages + t.rest + 2 * (size_t)t.nstage * 8 + (size_t)t.nstage * 4;
  return t;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

// One tensor map over a slot arena: dims / strides innermost first, the last dimension the slot. L2 promotion
// of 128 bytes, the width of a box row (32 words): wider promotion (256 bytes) fetched the neighbouring
// columns, which other CTAs load themselves, and cost 0.6 us per config-1 layer.
bool encode_map(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
                const cuuint64_t* strides, const cuuint32_t* box) {
  const cuuint32_t es[4] = {1, 1, 1, 1};
  return tensor_map_encoder()(m, dt, (cuuint32_t)rank, const_cast<void*>(base), dims, strides, box, es,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The six arena maps; cached per thread on everything they depend on (the arena never moves between
// decode steps, so steady-state calls encode nothing).
bool arena_maps(const LayerArgs& a, CUtensorMap (&tm)[6]) {
  struct Key {
    const void* b[6];
    int64_t st[6];
    int H, I, S;
    bool operator==(const Key& o) const {
      for (int k = 0; k < 6; ++k)
        if (b[k] != o.b[k] || st[k] != o.st[k]) return false;
      return H == o.H && I == o.I && S == o.S;
    }
  };
  static thread_local Key last{};
  static thread_local bool have = false;
  static thread_local CUtensorMap cache[6];
  const Key k{{a.map13.wbase, a.map13.sbase, a.map13.zbase, a.map2.wbase, a.map2.sbase, a.map2.zbase},
              {a.map13.wstride, a.map13.sstride, a.map13.zstride, a.map2.wstride, a.map2.sstride, a.map2.zstride},
              a.H, a.I, a.map13.S};
  if (!(have && last == k)) {
    have = false;
    if (!tensor_map_encoder()) return false;
    // the slot dimension is the arena's real slot count: a copy can never leave the arena
    const cuuint64_t I = (cuuint64_t)a.I, H = (cuuint64_t)a.H, S = (cuuint64_t)a.map13.S;
    const bool hz = a.map13.has_zeros != 0;
    {  // gate_up: (column within half, half, row, slot)
      const cuuint64_t dc[4] = {I, 2, H / 16, S}, sc[3] = {I * 4, 2 * I * 4, (cuuint64_t)a.map13.wstride};
      const cuuint32_t bc[4] = {32, 2, 16, 1};
      const cuuint64_t ds[4] = {I, 2, H / kGroup, S}, ss[3] = {I * 2, 2 * I * 2, (cuuint64_t)a.map13.sstride};
      const cuuint32_t bs[4] = {32, 2, 2, 1};
      if (!encode_map(&cache[0], CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, a.map13.wbase, dc, sc, bc)) return false;
      if (!encode_map(&cache[1], CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, a.map13.sbase, ds, ss, bs)) return false;
      if (hz) {
        const cuuint64_t dz[4] = {I / 4, 2, H / kGroup, S}, sz[3] = {I / 4, I / 2, (cuuint64_t)a.map13.zstride};
        const cuuint32_t bz[4] = {16, 2, 2, 1};
        if (!encode_map(&cache[2], CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, a.map13.zbase, dz, sz, bz)) return false;
      }
    }
    {  // down: (column, row, slot)
      const cuuint64_t dc[3] = {H, I / 16, S}, sc[2] = {H * 4, (cuuint64_t)a.map2.wstride};
      const cuuint32_t bc[3] = {32, 32, 1};
      const cuuint64_t ds[3] = {H, I / kGroup, S}, ss[2] = {H * 2, (cuuint64_t)a.map2.sstride};
      const cuuint32_t bs[3] = {32, 4, 1};
      if (!encode_map(&cache[3], CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, a.map2.wbase, dc, sc, bc)) return false;
      if (!encode_map(&cache[4], CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, a.map2.sbase, ds, ss, bs)) return false;
      if (hz) {
        const cuuint64_t dz[3] = {H / 4, I / kGroup, S}, sz[2] = {H / 4, (cuuint64_t)a.map2.zstride};
        const cuuint32_t bz[3] = {16, 4, 1};
        if (!encode_map(&cache[5], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, a.map2.zbase, dz, sz, bz)) return false;
      }
    }
    last = k;
    have = true;
  }
  for (int k2 = 0; k2 < 6; ++k2) tm[k2] = cache[k2];
  return true;
}

// Copy-engine mode needs a slot arena, 16-byte strides in every map (H and I multiples of 64) and the
// driver's tensor-map encoder.
bool tma_eligible(const LayerArgs& a) {
  if (a.map13.slots == nullptr || a.map2.slots == nullptr || a.map13.S <= 0 || a.map13.S != a.map2.S) return false;
  if (a.H % 64 != 0 || a.I % 64 != 0) return false;
  return tensor_map_encoder() != nullptr;
}

// The layer geometry of an M-token launch, with the slot table staged in shared memory when both
// projections share one that is small enough.
Geo layer_geo(const LayerArgs& a, int M, int grid_cap) {
  Geo g = make_geo(M, a.H, a.I, a.top_k, grid_cap);
  const bool shared = a.map13.slots != nullptr && a.map13.slots == a.map2.slots && a.map13.E == a.map2.E;
  g.stab = shared && a.map13.E > 0 && a.map13.E <= kMaxStagedSlots ? a.map13.E : 0;
  return g;
}

int launch_fused(const LayerArgs& a, int M, const void* x, const int32_t* ids, const float* w, void* y,
                        int grid_cap, bool tma) {
  const Geo g = layer_geo(a, M, grid_cap);
  const SmemPlan sp = smem_plan(g);
  FusedParams p{};
  p.x = static_cast<const __nv_bfloat16*>(x); p.ids = ids; p.topk_w = w;
  p.map13 = a.map13; p.map2 = a.map2; p.scale_bf16 = a.scale_bf16; p.rsf = a.routed_scaling;
  p.y = static_cast<__nv_bfloat16*>(y); p.geo = g; p.err = a.err;
  const PeerExchange* ex = a.xin ? a.xin : a.yout;
  if (ex) {
    p.xin = a.xin != nullptr;
    p.yout = a.yout != nullptr;
    p.xpeers = ex->peers; p.xtag_off = ex->tag_off; p.xn_max = ex->n_max; p.xrank = ex->rank;
    p.xworld = ex->world; p.xepoch = ex->epoch;
    p.xspin = ex->spin_limit ? ex->spin_limit : kPeerSpinLimit;
  }
  size_t base = 0, total = sp.total;
  if (tma) {
    const TmaPlan tp = tma_plan(g);
    if (tp.nstage == 0 || !arena_maps(a, p.tm)) return kErrShape;
    p.nstage = tp.nstage;
    p.off_stages = 0;
    base = tp.stages;
    p.off_bars = tp.stages + tp.rest;
    total = tp.total;
  }
  p.off_tabs = base;
  p.off_mail1 = base + sp.tabs;
  p.off_mail2 = p.off_mail1 + sp.mail1;
  p.off_rows = p.off_mail2 + sp.mail2;
  p.off_misc = p.off_rows + sp.rows;
  p.off_live = p.off_misc + sp.misc;
  p.off_slots = p.off_live + sp.live;
  p.off_preg = p.off_slots + sp.slots;
  unsigned* ctl = static_cast<unsigned*>(a.workspace);
  p.bar_count = ctl;
  p.bar_gen = ctl + 32;
  p.hand = reinterpret_cast<unsigned long long*>(static_cast<unsigned char*>(a.workspace) + 256);
  p.htab = static_cast<unsigned char*>(a.workspace) + 256 + kHandBytes;

  auto kern = ex ? (tma ? fused_layer_kernel<true, true> : fused_layer_kernel<false, true>)
                 : (tma ? fused_layer_kernel<true, false> : fused_layer_kernel<false, false>);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)total) != cudaSuccess)
    return kErrLaunch;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(g.grid);
  cfg.blockDim = dim3(tma ? kTmaThreads : kThreads);
  cfg.dynamicSmemBytes = total;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // start while the previous kernel ends
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, p) == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace

bool layer_arena_maps(const LayerArgs& a, CUtensorMap (&tm)[6]) { return tma_eligible(a) && arena_maps(a, tm); }

int decode_layer_fused(const LayerArgs& a) {
  if (a.M <= 0) return kOk;
  if (a.H % kGroup != 0 || a.I % kGroup != 0 || a.top_k <= 0) return kErrShape;
  if ((!a.x && !a.xin) || !a.ids || !a.topk_w || (!a.y && !a.yout)) return kErrArg;
  if (a.xin && a.yout && a.xin != a.yout) return kErrArg;        // one channel per layer
  if (const PeerExchange* ex = a.xin ? a.xin : a.yout) {
    if (!ex->peers || !ex->epoch || ex->world <= 0 || ex->rank < 0 || ex->rank >= ex->world || ex->n_max % 8 ||
        (size_t)a.M * a.H > (size_t)ex->n_max || ex->tag_off % 16)
      return kErrArg;
  }
  if (!a.workspace || a.workspace_bytes < layer_workspace_bytes(a.M, a.H, a.I, a.top_k)) return kErrWorkspace;
  if (reinterpret_cast<uintptr_t>(a.workspace) & 255u) return kErrAlign;

  static thread_local int cached_dev = -1, cached_cap = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kErrDevice;
  if (dev != cached_dev) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return kErrDevice;
    cached_cap = sms < kMaxGrid ? sms : kMaxGrid;   // one CTA per SM
    cached_dev = dev;
  }
  // tokens per launch: as many as the shared-memory plan allows (copy-engine mode also keeps a ring of
  // at least kMinStages stages)
  const bool tma = tma_eligible(a);
  auto fits = [&](int m) {
    const Geo g = layer_geo(a, m, cached_cap);
    return tma ? tma_plan(g).nstage > 0 : smem_plan(g).total <= 227 * 1024;
  };
  int mmax = a.M;
  while (mmax > 1 && !fits(mmax)) --mmax;
  if (!fits(mmax)) return kErrShape;
  if ((a.xin || a.yout) && mmax < a.M) return kErrShape;       // an exchange call is one launch
  for (int m0 = 0; m0 < a.M; m0 += mmax) {
    const int mc = a.M - m0 < mmax ? a.M - m0 : mmax;
    const int st = launch_fused(a, mc, static_cast<const __nv_bfloat16*>(a.x) + (size_t)m0 * a.H,
                                a.ids + (size_t)m0 * a.top_k, a.topk_w + (size_t)m0 * a.top_k,
                                static_cast<__nv_bfloat16*>(a.y) + (size_t)m0 * a.H, cached_cap, tma);
    if (st != kOk) return st;
  }
  return kOk;
}

}  // namespace w2a16
