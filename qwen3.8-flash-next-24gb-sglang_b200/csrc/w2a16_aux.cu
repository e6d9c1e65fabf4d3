// Load-time and arena kernels: bit-exact word relayout and the table-driven row gather.
#include "w2a16_kernels.h"

namespace w2a16 {

// dst[e][kw][n] = src32[e][n][kw]: the int32 view of the loader bytes [E, N, K/4] transposed per
// expert; the 4 bytes k/4 .. k/4+3 of row n become word k/16 of column n (little endian), exactly the
// byte move of gemv/moe_gemv_int2_tab.py:100-109.
__global__ void __launch_bounds__(256) to_word_ncontig_kernel(const uint32_t* __restrict__ src,
                                                              uint32_t* __restrict__ dst, int N, int KW) {
  __shared__ uint32_t tile[32][33];
  const int e = blockIdx.z;
  const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  const uint32_t* s = src + (int64_t)e * N * KW;
  uint32_t* d = dst + (int64_t)e * N * KW;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int n = n0 + i, k = k0 + threadIdx.x;
    if (n < N && k < KW) tile[i][threadIdx.x] = s[(int64_t)n * KW + k];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int k = k0 + i, n = n0 + threadIdx.x;
    if (n < N && k < KW) d[(int64_t)k * N + n] = tile[threadIdx.x][i];
  }
}

int to_word_ncontig(const void* src, void* dst, int E, int N, int K, cudaStream_t stream) {
  if (E <= 0 || N <= 0) return kOk;
  if (K <= 0 || K % 16 != 0) return kErrShape;
  if (!src || !dst) return kErrArg;
  if ((reinterpret_cast<uintptr_t>(src) & 3u) || (reinterpret_cast<uintptr_t>(dst) & 3u)) return kErrAlign;
  const int KW = K / 16;
  dim3 grid((N + 31) / 32, (KW + 31) / 32, E), block(32, 8);
  to_word_ncontig_kernel<<<grid, block, 0, stream>>>(static_cast<const uint32_t*>(src),
                                                     static_cast<uint32_t*>(dst), N, KW);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

// out[i, :] = row at tab[ids[i]] (patches/placement.py:34-43); 16-byte vectors.
__global__ void __launch_bounds__(256) gather_rows_tab_kernel(const int64_t* __restrict__ tab,
                                                              const int32_t* __restrict__ ids,
                                                              uint4* __restrict__ out, int64_t row_vec) {
  const int i = blockIdx.y;
  const uint4* src = reinterpret_cast<const uint4*>(tab[ids[i]]);
  uint4* dst = out + (int64_t)i * row_vec;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < row_vec; v += (int64_t)gridDim.x * blockDim.x)
    dst[v] = src[v];
}

int gather_rows_tab(const int64_t* tab, const int32_t* ids, int n, void* out, int64_t row_bytes,
                    cudaStream_t stream) {
  if (n <= 0 || row_bytes == 0) return kOk;
  if (!tab || !ids || !out) return kErrArg;
  if (row_bytes % 16 != 0 || (reinterpret_cast<uintptr_t>(out) & 15u)) return kErrAlign;
  const int64_t rv = row_bytes / 16;
  int bx = (int)((rv + 255) / 256);
  if (bx > 1024) bx = 1024;
  if (n > 65535) return kErrShape;
  gather_rows_tab_kernel<<<dim3(bx, n), 256, 0, stream>>>(tab, ids, static_cast<uint4*>(out), rv);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace w2a16
