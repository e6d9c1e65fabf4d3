// One-shot all-reduce (sum) of a small bf16 vector across the GPUs of one node over NVLink peer memory,
// for the expert-parallel decode step: every rank holds a partial MoE-layer output [M, H] (8 KB at M=1)
// and needs the sum.
//
// Buffers (push form): each rank owns a peer-visible buffer holding 2 parity slots x world x n_max bf16
// (slot p, row r = rank r's partial) and, at `flag_off` bytes, `world` flag words (zero before the first
// call); every rank maps every other rank's buffer (the caller passes a device array of the N peer addresses,
// e.g. from torch symmetric memory). Call e (a per-rank device counter, identical on all ranks because every
// rank makes the same calls) uses slot e & 1:
//   1. write the local partial into row my_rank of slot e & 1 of EVERY rank's buffer (NVLink stores);
//   2. one system-scope acq_rel fence after the CTA barrier, then store e into flag[my_rank] of every rank
//      (release);
//   3. wait until this rank's own flags hold e or later from every rank (acquire, bounded; signed distance,
//      because a faster rank may already have finished call e and raised its flag to e + 1);
//   4. sum the world rows of this rank's own slot in rank order 0..N-1 in fp32 -> bf16 out (local reads;
//      the same order on every rank, so every rank gets bit-identical sums).
// A rank writes call e's rows only after it saw every rank's call e-1 flag, which each rank raises only
// after it finished reading call e-2's slot, the one call e overwrites. Plain loads and stores to peer
// memory only; no multicast.
#include "w2a16_kernels.h"

namespace w2a16 {
namespace {

constexpr unsigned kArSpinLimit = 1u << 22;                  // default polls before a flag wait gives up
constexpr int kArThreads = 512;

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct ArParams {
  const __nv_bfloat16* in;
  __nv_bfloat16* out;
  int n, n_max, rank, world;
  const uint64_t* bufs;   // [world] peer buffer addresses (bf16 [2][world][n_max], flags at flag_off)
  size_t flag_off;
  unsigned* epoch;        // this rank's call counter
  unsigned* err;
  unsigned spin_limit;    // polls before a flag wait gives up
};

__global__ void __launch_bounds__(kArThreads, 1) allreduce_kernel(ArParams p) {
  // the next kernel of the stream (the INT8 projection, launched with programmatic stream serialisation)
  // may start its weight loads now; it waits for this grid before it reads the sum
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  __shared__ unsigned s_epoch;
  if (threadIdx.x == 0) s_epoch = *p.epoch + 1u;
  __syncthreads();
  const unsigned e = s_epoch;
  const size_t slot = (size_t)(e & 1u) * p.world * p.n_max;
  const size_t row = slot + (size_t)p.rank * p.n_max;
  // 16-byte pieces of the partial pushed to every rank (n is a multiple of 8)
  const int n8 = p.n / 8;
  for (int i = threadIdx.x; i < n8 * p.world; i += blockDim.x) {
    const int r = i / n8, k = i - r * n8;
    const uint4 v = reinterpret_cast<const uint4*>(p.in)[k];
    reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.bufs[r]) + row)[k] = v;
  }
  __syncthreads();
  if (threadIdx.x < p.world) {
    asm volatile("fence.acq_rel.sys;\n" ::: "memory");
    unsigned* peer_flags = reinterpret_cast<unsigned*>(p.bufs[threadIdx.x] + p.flag_off);
    st_release_sys(peer_flags + p.rank, e);
    const unsigned* own_flags = reinterpret_cast<const unsigned*>(p.bufs[p.rank] + p.flag_off);
    unsigned it = 0;
    // rank threadIdx.x's call-e row is in place once its flag reached e: a flag already at e + 1 means that
    // rank finished call e too (it cannot reach e + 2 before this rank has read call e's slot)
    while ((int)(ld_acquire_sys(own_flags + threadIdx.x) - e) < 0) {
      if (++it > p.spin_limit) {
        flag_error(p.err, 2u);
        break;
      }
    }
  }
  __syncthreads();
  const __nv_bfloat16* mine = reinterpret_cast<const __nv_bfloat16*>(p.bufs[p.rank]) + slot;
  for (int i = threadIdx.x; i < p.n; i += blockDim.x) {
    float acc = 0.f;
    for (int r = 0; r < p.world; ++r) acc += __bfloat162float(mine[(size_t)r * p.n_max + i]);
    p.out[i] = __float2bfloat16(acc);
  }
  if (threadIdx.x == 0) *p.epoch = e;
}

}  // namespace

int allreduce_peers_bf16(const void* in, void* out, int n, int n_max, const uint64_t* bufs, size_t flag_off, int rank,
                         int world, unsigned* epoch, unsigned* err, unsigned spin_limit, cudaStream_t stream) {
  if (n <= 0) return kOk;
  if (!in || !out || !bufs || !epoch || world <= 0 || world > kArThreads || rank < 0 || rank >= world)
    return kErrArg;
  if (n > n_max || n % 8 || n_max % 8 || flag_off < (size_t)n_max * 4 * world || flag_off % 16) return kErrShape;
  if ((reinterpret_cast<uintptr_t>(in) & 15u)) return kErrAlign;
  ArParams p{};
  p.in = static_cast<const __nv_bfloat16*>(in);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.n = n; p.n_max = n_max; p.rank = rank; p.world = world;
  p.bufs = bufs; p.flag_off = flag_off; p.epoch = epoch; p.err = err;
  p.spin_limit = spin_limit ? spin_limit : kArSpinLimit;
  allreduce_kernel<<<1, kArThreads, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace w2a16
