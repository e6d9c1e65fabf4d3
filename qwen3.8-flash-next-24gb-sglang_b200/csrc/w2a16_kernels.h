// Internal host-side declarations shared by the kernel translation units and the C ABI layer.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include "w2a16_common.cuh"

namespace w2a16 {

struct GemvArgs {
  const void* a;
  int64_t stride_am;
  ExpertMap map;
  const int32_t* ids;
  const float* topk_w;
  void* out;
  int64_t stride_om;
  int R, N, K, top_k;
  int64_t stride_ww, stride_sg, stride_zg;
  int mul_routed_weight;
  int scale_bf16;
  unsigned* err;
  cudaStream_t stream;
};

int gemv_plain(const GemvArgs& g);

// Exchange channel between the ranks of an expert-parallel step: every rank's peer-visible buffer holds, at
// tag_off bytes, 2 parity slots x world rows x n_max / 2 tagged words -- word j of row r carries values 2j and
// 2j + 1 (bf16) of rank r's partial of a call with that parity in its low 32 bits and the call number in its high
// 32 bits (one single-copy-atomic 8-byte store, so a reader that sees the call number sees the data). Call e
// uses slot e & 1; *epoch counts the channel's calls on this rank.
struct PeerExchange {
  const uint64_t* peers;  // device array [world] of the peer buffer addresses
  size_t tag_off;
  int n_max, rank, world;
  unsigned* epoch;        // calls made on this channel (device word)
  unsigned spin_limit;    // polls of a word before a wait gives up (0: the library default)
};

// Fused persistent decode layer (w2a16_layer.cu).
struct LayerArgs {
  const void* x;          // bf16 [M, H]
  int M, H, I, top_k;
  const int32_t* ids;     // [M * top_k]
  const float* topk_w;    // [M * top_k]
  ExpertMap map13;        // gate_up: codes [H/16, 2I], scales [H/128, 2I], zeros [H/128, 2I/4]
  ExpertMap map2;         // down:    codes [I/16, H],  scales [I/128, H],  zeros [I/128, H/4]
  int scale_bf16;
  float routed_scaling;
  void* y;                // bf16 [M, H]
  void* workspace;
  size_t workspace_bytes;
  unsigned* err;
  cudaStream_t stream;
  // expert parallelism: x = the sum of the ranks' rows of the channel's call *epoch (instead of x), and/or this
  // layer's partial pushed as this rank's row of call *epoch + 1 (instead of y)
  const PeerExchange* xin = nullptr;
  const PeerExchange* yout = nullptr;
};
size_t layer_workspace_bytes(int M, int H, int I, int top_k);
int decode_layer_fused(const LayerArgs& a);
// The six arena tensor maps of the fused layer's copy-engine mode (gate_up codes / scales / zeros, then
// down); false when the arena does not qualify (no slot table, H or I not a multiple of 64, no encoder).
bool layer_arena_maps(const LayerArgs& a, CUtensorMap (&tm)[6]);

// Batched layer on the tensor cores (w2a16_grouped.cu): M >= kGroupedMinTokens, slot arenas only. The C ABI's
// automatic choice takes it from W2A16_BATCHED_AUTO_TOKENS tokens, where it is the faster one.
constexpr int kGroupedMinTokens = 16;
size_t grouped_workspace_bytes(int M, int H, int I, int top_k);
// kOk when the grouped path can take this call; kErrShape (token count, table form or shape), kErrAlign or
// kErrWorkspace (the workspace does not hold its buffers) otherwise.
int grouped_check(const LayerArgs& a);
int decode_layer_grouped(const LayerArgs& a);
int allreduce_peers_bf16(const void* in, void* out, int n, int n_max, const uint64_t* bufs, size_t flag_off, int rank,
                         int world, unsigned* epoch, unsigned* err, unsigned spin_limit, cudaStream_t stream);

// INT8 dense GEMV (w2a16_int8.cu).
struct Int8Args {
  const void* x;          // bf16 [M, K]
  int64_t stride_xm;
  const int32_t* qweight; // int32 [K/4, N], 4 uint8 along K per word
  const void* scales;     // f16 [K/g, N]
  int group;              // K for per-output-channel scales
  int zero;               // 128 = symmetric
  int M, K, N;
  void* y;                // bf16 [M, N]
  int64_t stride_ym;
  cudaStream_t stream;
};
int int8_gemv(const Int8Args& a, void* workspace, size_t workspace_bytes);
// The same with x the sum of the ranks' rows of the channel's call *epoch (M * K <= n_max).
int int8_gemv_from_peers(const Int8Args& a, const PeerExchange& xin, unsigned* err);
size_t int8_workspace_bytes(int M, int K, int N);
int to_word_ncontig(const void* src, void* dst, int E, int N, int K, cudaStream_t stream);
int gather_rows_tab(const int64_t* tab, const int32_t* ids, int n, void* out, int64_t row_bytes, cudaStream_t stream);

}  // namespace w2a16
