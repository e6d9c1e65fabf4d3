// Shared device code for the W2A16 group-128 MoE GEMV kernels (sm_100a).
//
// Weight layout (the reference's N-contiguous int32-word layout, gemv/moe_gemv_int2_tab.py:3-5):
//   codes  uint32 [K/16, N] per expert: value k of column n at bits 2*(k%16) of word k/16
//   scales f16|bf16 [K/128, N] per expert
//   zeros  uint8 [K/128, N/4] per expert (optional): zero point of column n at bits 2*(n%4) of byte
//          n/4; absent -> symmetric zero point 2 (gemv/moe_gemv_int2_tab.py:66)
//
// Inner product on CUDA cores with integer dot-product instructions:
//   * a word holds 16 codes; the mask w & (0x03030303 << 2j) ("class j") leaves four bytes holding
//     q*4^j for codes j, j+4, j+8, j+12 -- one LOP3 per 4 codes, no shifts;
//   * the activation of each 128-wide group is held as 16-bit fixed point x_fixed = x / 2^e_g
//     (power-of-two group scale, |x_fixed| <= 32767, exact for every bf16 value within 2^8 of the
//     group maximum), packed in pairs so that dp2a.lo / dp2a.hi multiply two code bytes by two
//     16-bit activations and accumulate exactly in int32;
//   * per (column, group): T = sum_j acc_j * 4^(3-j) = 64 * sum_k q_k x_fixed_k, the zero point is
//     folded as T - 64 * zp * sum_k x_fixed_k (the reference folds it the same way,
//     gemv/moe_gemv_int2_tab.py:61-66), then one I2F and one FFMA with s * 2^(e_g - 6) move the
//     group into the fp32 accumulator.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace w2a16 {

constexpr int kGroup = 128;        // quantization group along K
constexpr int kWordsPerGroup = 8;  // 128 codes / 16 codes per word
constexpr int kXRegs = 8;          // packed activation registers per word row (4 classes x lo/hi)

// Status codes shared with the C ABI (include/w2a16_moe.h).
enum Status : int {
  kOk = 0,
  kErrShape = 1,
  kErrAlign = 2,
  kErrLaunch = 3,
  kErrArg = 4,
  kErrWorkspace = 5,
  kErrDevice = 6,
  kErrMemory = 7,
};

// Device-side error word: bit 0 = an expert id outside [0, E) or an arena slot id outside [-1, S) (the row
// contributes zero), bit 1 = a bounded wait gave up, bit 2 = a misaligned shared-memory ring (copies skipped).
__device__ __forceinline__ void flag_error(unsigned* err, unsigned bit) {
  if (err) atomicOr(err, bit);
}

// ----------------------------------------------------------------------------- peer exchange (expert parallelism)
constexpr unsigned kPeerSpinLimit = 1u << 22;   // default polls before a peer flag wait gives up

__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys_u32(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_relaxed_gpu_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Tagged exchange words: (call << 32) | (two bf16 values), written and read as one 8-byte access each.
__device__ __forceinline__ void st_tagged(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}
// The data of word w of call e, once it holds that call. `budget` is the calling thread's poll allowance for all
// the words it reads (bounded: when it runs out, bit 1 of err and the stale data -- every later word is then
// looked at once). A writer stores call e + 2 into the same word only after this rank has finished reading call e.
__device__ __forceinline__ uint32_t wait_tagged(const unsigned long long* w, unsigned e, unsigned& budget,
                                                unsigned* err) {
  unsigned long long v;
  for (;;) {
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];\n" : "=l"(v) : "l"(w) : "memory");
    if ((unsigned)(v >> 32) == e) break;
    if (budget == 0) {
      flag_error(err, 2u);
      break;
    }
    --budget;
  }
  return (uint32_t)v;
}
// bf16 pair -> two floats
__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
}

// ----------------------------------------------------------------------------- integer dot products
__device__ __forceinline__ int dp2a_lo(uint32_t a16x2, uint32_t b8x4, int c) {
  int d;
  asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a16x2), "r"(b8x4), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_hi(uint32_t a16x2, uint32_t b8x4, int c) {
  int d;
  asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a16x2), "r"(b8x4), "r"(c));
  return d;
}

// acc[j] += sum over the 16 codes of word w of (q*4^j) * x_fixed, for the class-j codes.
// xr = the 8 packed activation registers of this word row.
__device__ __forceinline__ void word_dot(uint32_t w, const uint32_t (&xr)[kXRegs], int (&acc)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t m = w & (0x03030303u << (2 * j));
    acc[j] = dp2a_lo(xr[2 * j], m, acc[j]);
    acc[j] = dp2a_hi(xr[2 * j + 1], m, acc[j]);
  }
}

// T = 64 * sum q x_fixed (exact): acc_j holds 4^j * partial sums.
__device__ __forceinline__ int combine_classes(const int (&acc)[4]) {
  return ((acc[0] * 4 + acc[1]) * 4 + acc[2]) * 4 + acc[3];
}

// ----------------------------------------------------------------------------- activation tables
// Per activation row: packed pairs [K/16][8] (uint32), per group: m64X = -64 * sum x_fixed,
// scl = 2^(e_g - 6). Index of element c (0..15) of word row kw: register j*2+h with j = c%4,
// h = c/8, half (c/4)%2, so register (j, h) = (x[j + 8h], x[j + 4 + 8h]) as (lo, hi) 16-bit halves.
struct XTable {
  uint32_t* pairs;  // [K/16 * 8]
  int* m64x;        // [K/128]
  float* scl;       // [K/128]
};

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }

// Exact power-of-two helpers: the frexp exponent E of a positive finite m (m = f * 2^E, f in [0.5, 1)),
// read from the float's exponent field, and 2^k built the same way; both fall back to the library
// functions only outside the normal range.
__device__ __forceinline__ int frexp_exponent(float m) {
  const int be = (int)((__float_as_uint(m) >> 23) & 0xFFu);
  if (be != 0) return be - 126;
  int E = 0;
  frexpf(m, &E);
  return E;
}
__device__ __forceinline__ float pow2f(int k) {
  return (k >= -126 && k <= 127) ? __uint_as_float((unsigned)(k + 127) << 23) : ldexpf(1.f, k);
}

// One warp converts one 128-value group of an activation row (src points at the group's first
// element). Lane l owns elements 4l .. 4l+3.
template <typename T>
__device__ __forceinline__ void prep_group_warp(const T* __restrict__ src, int g, XTable tab, int lane) {
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = to_f32<T>(src[4 * lane + i]);
  float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  // mx = f * 2^E with f in [0.5, 1) -> x / 2^(E-15) lies in (-32768, 32768)
  const int e = (mx > 0.f ? frexp_exponent(mx) : 0) - 15;
  const float inv = pow2f(-e);
  int s = 0;
  uint16_t* half = reinterpret_cast<uint16_t*>(tab.pairs);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int q = __float2int_rn(v[i] * inv);
    q = max(-32767, min(32767, q));
    s += q;
    const int k = g * kGroup + 4 * lane + i;  // position within the row
    const int kw = k >> 4, c = k & 15;
    const int reg = (c & 3) * 2 + (c >> 3);
    const int hf = (c >> 2) & 1;
    half[(kw * kXRegs + reg) * 2 + hf] = static_cast<uint16_t>(q);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) {
    tab.m64x[g] = -64 * s;
    tab.scl[g] = pow2f(e - 6);
  }
}

// NG groups at once, with their lane reductions interleaved (the same conversion as prep_group_regs):
// lane l holds elements 4l .. 4l+3 of group gl[j] in v[j]; group j goes to the table of a K-long row
// that starts toff[j] bytes after `base` (pairs, then m64x, then scl); groups with gl[j] < 0 are
// skipped. Lane pairs (2i, 2i+1) hold the two 16-bit halves of the same packed register, so even lanes
// store whole words.
template <int NG>
__device__ __forceinline__ void prep_groups(const float (&v)[NG][4], const int (&gl)[NG], const int (&toff)[NG],
                                            unsigned char* base, int K, int lane) {
  float mx[NG];
#pragma unroll
  for (int j = 0; j < NG; ++j)
    mx[j] = fmaxf(fmaxf(fabsf(v[j][0]), fabsf(v[j][1])), fmaxf(fabsf(v[j][2]), fabsf(v[j][3])));
  // |x| of a non-negative float orders like its bit pattern: one integer max reduction per group
#pragma unroll
  for (int j = 0; j < NG; ++j) mx[j] = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(mx[j])));
  int e[NG], s[NG], q[NG][4];
#pragma unroll
  for (int j = 0; j < NG; ++j) {
    e[j] = (mx[j] > 0.f ? frexp_exponent(mx[j]) : 0) - 15;
    const float inv = pow2f(-e[j]);
    s[j] = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      q[j][i] = max(-32767, min(32767, __float2int_rn(v[j][i] * inv)));
      s[j] += q[j][i];
    }
  }
  // element 4l+i of the group: word row l/4, register 2i + (l%4)/2, half l%2
#pragma unroll
  for (int j = 0; j < NG; ++j) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int other = __shfl_xor_sync(0xffffffffu, q[j][i], 1);
      if (gl[j] >= 0 && (lane & 1) == 0) {
        const uint32_t word = (uint32_t)(q[j][i] & 0xFFFF) | ((uint32_t)other << 16);
        reinterpret_cast<uint32_t*>(base + toff[j])[(gl[j] * 8 + (lane >> 2)) * kXRegs + 2 * i + ((lane & 3) >> 1)] =
            word;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NG; ++j) s[j] = __reduce_add_sync(0xffffffffu, s[j]);
  if (lane == 0) {
#pragma unroll
    for (int j = 0; j < NG; ++j)
      if (gl[j] >= 0) {
        int* m64x = reinterpret_cast<int*>(base + toff[j] + (size_t)(K / 16) * kXRegs * 4);
        m64x[gl[j]] = -64 * s[j];
        reinterpret_cast<float*>(m64x + K / kGroup)[gl[j]] = pow2f(e[j] - 6);
      }
  }
}

// The conversion for values already in registers: lane l holds elements 4l .. 4l+3 of group `gl`.
__device__ __forceinline__ void prep_group_regs(const float (&v)[4], int gl, XTable tab, int lane) {
  float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const int e = (mx > 0.f ? frexp_exponent(mx) : 0) - 15;
  const float inv = pow2f(-e);
  int s = 0;
  uint16_t* half = reinterpret_cast<uint16_t*>(tab.pairs);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int q = __float2int_rn(v[i] * inv);
    q = max(-32767, min(32767, q));
    s += q;
    const int k = gl * kGroup + 4 * lane + i;
    const int kw = k >> 4, c = k & 15;
    half[(kw * kXRegs + (c & 3) * 2 + (c >> 3)) * 2 + ((c >> 2) & 1)] = static_cast<uint16_t>(q);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) {
    tab.m64x[gl] = -64 * s;
    tab.scl[gl] = pow2f(e - 6);
  }
}

// ----------------------------------------------------------------------------- expert addressing
// Either the reference's int64 address tables (make_tables, gemv/moe_gemv_int2_tab.py:88-97) or the
// arena form: base + slot[e] * stride, slot -1 = expert not resident -> the row contributes zero. An arena
// holds S slots; a slot id of S or more is treated like -1 and sets bit 0 of the error word, so a corrupt
// slot table never reads past the arena.
struct ExpertMap {
  const int64_t* wtab;
  const int64_t* stab;
  const int64_t* ztab;
  const int32_t* slots;
  const char* wbase;
  const char* sbase;
  const char* zbase;
  int64_t wstride;  // bytes per slot
  int64_t sstride;
  int64_t zstride;
  int E;
  int S;            // arena slots (slot form only)
  int has_zeros;

  __device__ __forceinline__ bool resolve(int e, const uint32_t*& w, const char*& s, const uint8_t*& z,
                                          unsigned* err) const {
    if (e < 0 || e >= E) {
      flag_error(err, 1u);
      return false;
    }
    if (slots != nullptr) {
      const int sl = slots[e];
      if (sl < 0) return false;
      if (sl >= S) {
        flag_error(err, 1u);
        return false;
      }
      w = reinterpret_cast<const uint32_t*>(wbase + (int64_t)sl * wstride);
      s = sbase + (int64_t)sl * sstride;
      z = has_zeros ? reinterpret_cast<const uint8_t*>(zbase + (int64_t)sl * zstride) : nullptr;
    } else {
      w = reinterpret_cast<const uint32_t*>(wtab[e]);
      s = reinterpret_cast<const char*>(stab[e]);
      z = has_zeros ? reinterpret_cast<const uint8_t*>(ztab[e]) : nullptr;
    }
    return true;
  }

  // Arena form with the slot of expert e already looked up (e in [0, E) checked by the caller).
  __device__ __forceinline__ bool resolve_slot(int sl, const uint32_t*& w, const char*& s, const uint8_t*& z,
                                               unsigned* err) const {
    if (sl < 0) return false;
    if (sl >= S) {
      flag_error(err, 1u);
      return false;
    }
    w = reinterpret_cast<const uint32_t*>(wbase + (int64_t)sl * wstride);
    s = sbase + (int64_t)sl * sstride;
    z = has_zeros ? reinterpret_cast<const uint8_t*>(zbase + (int64_t)sl * zstride) : nullptr;
    return true;
  }
};

__device__ __forceinline__ float load_scale(const char* sptr, int64_t idx, bool bf16) {
  if (bf16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(sptr)[idx]);
  return __half2float(reinterpret_cast<const __half*>(sptr)[idx]);
}

// 4 consecutive scales (8 bytes, 8-byte aligned) -> fp32
__device__ __forceinline__ void load_scale4(const char* sptr, int64_t idx, bool bf16, float (&s)[4]) {
  const uint2 raw = *reinterpret_cast<const uint2*>(sptr + idx * 2);
  if (bf16) {
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
    s[0] = __low2float(a); s[1] = __high2float(a); s[2] = __low2float(b); s[3] = __high2float(b);
  } else {
    const __half2 a = *reinterpret_cast<const __half2*>(&raw.x);
    const __half2 b = *reinterpret_cast<const __half2*>(&raw.y);
    s[0] = __low2float(a); s[1] = __high2float(a); s[2] = __low2float(b); s[3] = __high2float(b);
  }
}

__device__ __forceinline__ float silu(float v) { return v / (1.f + __expf(-v)); }

}  // namespace w2a16
