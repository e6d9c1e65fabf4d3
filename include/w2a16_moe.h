/*
 * w2a16_moe.h — C ABI of the B200 (sm_100a) W2A16 group-128 MoE decode GEMV library.
 *
 * Plain pointers and sizes only. Every device pointer is a CUDA device address (or a pinned host
 * address reachable through unified addressing, where noted). Every entry point that launches
 * work takes a cudaStream_t passed as `void* stream` (NULL = legacy default stream), performs no
 * host synchronisation and no allocation, and returns a status code:
 *
 *   0 W2A16_OK            success (kernels enqueued)
 *   1 W2A16_ERR_SHAPE     a dimension is not supported (K % 128, N % 4, ...)
 *   2 W2A16_ERR_ALIGN     a stride or base address breaks the 16-byte rule
 *   3 W2A16_ERR_LAUNCH    the CUDA launch failed (cudaGetLastError)
 *   4 W2A16_ERR_ARG       a required pointer is NULL or an argument is out of range
 *   5 W2A16_ERR_WORKSPACE the workspace is missing or too small
 *   6 W2A16_ERR_DEVICE    no usable sm_100 device
 *   7 W2A16_ERR_MEMORY    no physical memory (or host memory) for another arena chunk
 *
 * Layouts (the reference's N-contiguous int32-word layout, gemv/moe_gemv_int2_tab.py:3-5):
 *   codes   int32 [K/16, N] per expert; value k of column n at bits 2*(k%16) of word k/16
 *   scales  f16 or bf16 [K/128, N] per expert (scale_bf16 selects bf16)
 *   zeros   uint8 [K/128, N/4] per expert, optional: zero point of column n at bits 2*(n%4) of
 *           byte n/4. Without zeros the symmetric zero point 2 applies (gemv/moe_gemv_int2_tab.py:66)
 *   w = (q - zp) * s.
 *
 * Device-side error word (`err`, optional, uint32 in device memory): bit 0 is set when an expert id
 * lies outside [0, num_experts), or when a slot table entry is num_slots or more (negative entries
 * mean "not resident" and are not errors); such rows contribute zero and nothing outside the arena is
 * read. Bit 1 is set when a bounded wait inside a kernel gave up. Bit 2 is set when the decode layer's
 * shared-memory ring is not 128-byte aligned (its copies are then skipped). The library never traps or
 * aborts.
 */
#ifndef W2A16_MOE_H
#define W2A16_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define W2A16_OK 0
#define W2A16_ERR_SHAPE 1
#define W2A16_ERR_ALIGN 2
#define W2A16_ERR_LAUNCH 3
#define W2A16_ERR_ARG 4
#define W2A16_ERR_WORKSPACE 5
#define W2A16_ERR_DEVICE 6
#define W2A16_ERR_MEMORY 7

/* Library version string, e.g. "w2a16_moe 0.1 sm_100a". */
const char* w2a16_version(void);

/* Human-readable name of a status code. */
const char* w2a16_status_string(int status);

/*
 * Batch-1 MoE GEMV through int64 address tables.
 * Replaces moe_gemv_int2_tab() — gemv/moe_gemv_int2_tab.py:72-85 (kernel :23-69), called from
 * MoeWNA16Method._apply_gemv (patches/ncontig_gemv.py:229, :232).
 *
 *   c[r, n] = (mul_routed_weight ? topk_w[r] : 1)
 *             * sum_k (q - zp) * s  of expert topk_ids[r], column n, times a[r / top_k, k]
 *
 * a        bf16 [*, K], row stride stride_am (elements)
 * wtab     int64 [num_experts] base address of each expert's codes  (make_tables, :88-97)
 * stab     int64 [num_experts] base address of each expert's scales
 * ztab     int64 [num_experts] base address of each expert's zeros, or NULL (symmetric, zp = 2)
 * topk_ids int32 [R] original expert ids; topk_w fp32 [R] (may be NULL if !mul_routed_weight)
 * c        bf16 [R, N], row stride stride_cm (elements); written, never read
 * stride_ww words per K/16 row of codes; stride_sg elements per scale row; stride_zg bytes per
 *          zero row. K % 128 == 0, N % 4 == 0, strides multiples of 4, bases 16-byte aligned.
 */
int w2a16_moe_gemv_tab(const void* a, int64_t stride_am,
                       const int64_t* wtab, const int64_t* stab, const int64_t* ztab, int num_experts,
                       const int32_t* topk_ids, const float* topk_w,
                       void* c, int64_t stride_cm,
                       int R, int N, int K,
                       int64_t stride_ww, int64_t stride_sg, int64_t stride_zg,
                       int top_k, int mul_routed_weight, int scale_bf16,
                       unsigned int* err, void* stream);

/*
 * The same GEMV over an expert arena addressed through an int32 slot table.
 * Replaces the int64 address-table indirection of RowArena / ExpertElastic
 * (gemv/row_arena.py:34-123, table writes gemv/expert_elastic.py:157, :220, :242;
 * placed tables patches/placement.py:208-227): expert e lives at
 *   codes_base  + slots[e] * codes_slot_bytes   (likewise scales, zeros)
 * and slots[e] == -1 marks a non-resident expert whose rows contribute zero. The arena holds
 * num_slots slots; an entry of num_slots or more is treated like -1 and sets bit 0 of `err`.
 */
int w2a16_moe_gemv_slots(const void* a, int64_t stride_am,
                         const int32_t* slots, int num_experts, int num_slots,
                         const void* codes_base, int64_t codes_slot_bytes,
                         const void* scales_base, int64_t scales_slot_bytes,
                         const void* zeros_base, int64_t zeros_slot_bytes,
                         const int32_t* topk_ids, const float* topk_w,
                         void* c, int64_t stride_cm,
                         int R, int N, int K,
                         int top_k, int mul_routed_weight, int scale_bf16,
                         unsigned int* err, void* stream);

/* Workspace bytes the decode-layer entry points need for M tokens (h buffer + control words). */
size_t w2a16_moe_layer_workspace_bytes(int M, int H, int I, int top_k);

/*
 * No counterpart in the reference (its batched path is the same Triton GEMV per routed row).
 * Workspace bytes of the batched path for M tokens (M >= 16): the routed rows grouped by expert, every
 * resident expert streamed once for all of its rows, the products on the tensor cores (route tables,
 * h [rows, I] bf16 and y rows [rows, H] fp32 for up to 128 tokens at a time), never less than
 * w2a16_moe_layer_workspace_bytes. Below 16 tokens it returns w2a16_moe_layer_workspace_bytes. The
 * batched path keeps out of the per-token path's persistent workspace words, so one workspace serves
 * calls of either path.
 */
size_t w2a16_moe_layer_workspace_bytes_batched(int M, int H, int I, int top_k);

/* Path choice of the slot-table decode layer (w2a16_moe_decode_layer_slots_ex). AUTO follows the token
 * count: the per-token path below W2A16_BATCHED_AUTO_TOKENS tokens, the batched path from there on when the
 * workspace holds its buffers (else the per-token path). BATCHED takes the batched path from 16 tokens and
 * returns W2A16_ERR_WORKSPACE when the workspace is too small for it (W2A16_ERR_SHAPE below 16 tokens or for
 * shapes it does not support). PER_TOKEN always takes the per-token path. */
#define W2A16_PATH_AUTO 0
#define W2A16_PATH_PER_TOKEN 1
#define W2A16_PATH_BATCHED 2
#define W2A16_BATCHED_AUTO_TOKENS 64

/*
 * Full decode MoE layer: gate_up GEMV, SiLU(gate) * up, down GEMV * routed weight, sum over the
 * top-k experts of each token, times routed_scaling_factor.
 * Replaces MoeWNA16Method._apply_gemv — patches/ncontig_gemv.py:218-238 (serving patch:3358-3400):
 * the two moe_gemv_int2_tab launches, the torch SiLU*mul and the torch top-k sum.
 *
 * x        bf16 [M, H] (row stride H); y bf16 [M, H] output
 * topk_ids int32 [M * top_k], topk_w fp32 [M * top_k] (token-major)
 * gate_up expert tensors: codes [H/16, 2I], scales [H/128, 2I], zeros [H/128, 2I/4] or NULL;
 *          rows [0, I) are gate, [I, 2I) are up (gemv/test_gemv_tab.py:32)
 * down expert tensors:    codes [I/16, H],  scales [I/128, H],  zeros [I/128, H/4] or NULL
 * workspace >= w2a16_moe_layer_workspace_bytes(); it must be zero-filled before its first use and
 *          is left zero-filled in its control words by every call.
 * H % 128 == 0, I % 128 == 0.
 */
int w2a16_moe_decode_layer_tab(const void* x, int M, int H, int I, int top_k,
                               const int32_t* topk_ids, const float* topk_w, int num_experts,
                               const int64_t* wtab13, const int64_t* stab13, const int64_t* ztab13,
                               const int64_t* wtab2, const int64_t* stab2, const int64_t* ztab2,
                               int scale_bf16, float routed_scaling_factor,
                               void* y, void* workspace, size_t workspace_bytes,
                               unsigned int* err, void* stream);

/* The decode layer over an int32 slot table into expert arenas of num_slots slots (slot -1 = not resident;
 * an entry of num_slots or more is treated like -1 and sets bit 0 of `err`). Path choice W2A16_PATH_AUTO. */
int w2a16_moe_decode_layer_slots(const void* x, int M, int H, int I, int top_k,
                                 const int32_t* topk_ids, const float* topk_w,
                                 const int32_t* slots, int num_experts, int num_slots,
                                 const void* codes13, int64_t codes13_slot_bytes,
                                 const void* scales13, int64_t scales13_slot_bytes,
                                 const void* zeros13, int64_t zeros13_slot_bytes,
                                 const void* codes2, int64_t codes2_slot_bytes,
                                 const void* scales2, int64_t scales2_slot_bytes,
                                 const void* zeros2, int64_t zeros2_slot_bytes,
                                 int scale_bf16, float routed_scaling_factor,
                                 void* y, void* workspace, size_t workspace_bytes,
                                 unsigned int* err, void* stream);

/* w2a16_moe_decode_layer_slots with an explicit path choice (W2A16_PATH_*); no counterpart in the reference. */
int w2a16_moe_decode_layer_slots_ex(const void* x, int M, int H, int I, int top_k,
                                    const int32_t* topk_ids, const float* topk_w,
                                    const int32_t* slots, int num_experts, int num_slots,
                                    const void* codes13, int64_t codes13_slot_bytes,
                                    const void* scales13, int64_t scales13_slot_bytes,
                                    const void* zeros13, int64_t zeros13_slot_bytes,
                                    const void* codes2, int64_t codes2_slot_bytes,
                                    const void* scales2, int64_t scales2_slot_bytes,
                                    const void* zeros2, int64_t zeros2_slot_bytes,
                                    int scale_bf16, float routed_scaling_factor,
                                    void* y, void* workspace, size_t workspace_bytes, int path,
                                    unsigned int* err, void* stream);

/*
 * No counterpart in the reference: this entry point exists only in this library.
 *
 * The decode layer over a slot table (same arguments and result as w2a16_moe_decode_layer_slots) for
 * callers that cannot allocate device memory and so cannot hand in a workspace: a host that reaches
 * this call while its stream is being captured into a CUDA graph (cudaMalloc is not allowed during a
 * global-mode capture), or a serving process whose device memory is fully reserved by its own pool at
 * start-up. It calls no cudaMalloc, cudaFree or allocating library routine. Its workspace is a fixed
 * array of W2A16_NOALLOC_SCRATCH_BYTES (4 MiB) inside the library that every GPU loading the library
 * holds until the process exits; layers needing more (w2a16_moe_layer_workspace_bytes(M, H, I, top_k)
 * > W2A16_NOALLOC_SCRATCH_BYTES; at I=1536, top-8 that is M > 146) return W2A16_ERR_WORKSPACE.
 * The first call in each CUDA context (once per device, and again after a device reset, which makes a
 * new context) looks up that array's device address for the calling thread's current device (which must
 * own `stream`); make that first call before any stream capture. The path choice is the one of
 * w2a16_moe_decode_layer_slots with this much workspace (per-token below W2A16_BATCHED_AUTO_TOKENS tokens).
 * All calls share the one array: calls that overlap on the GPU (different streams, or concurrent graph replays) race
 * and must not be issued.
 */
#define W2A16_NOALLOC_SCRATCH_BYTES (4u << 20)
int w2a16_moe_decode_layer_slots_noalloc(const void* x, int M, int H, int I, int top_k,
                                         const int32_t* topk_ids, const float* topk_w,
                                         const int32_t* slots, int num_experts, int num_slots,
                                         const void* codes13, int64_t codes13_slot_bytes,
                                         const void* scales13, int64_t scales13_slot_bytes,
                                         const void* zeros13, int64_t zeros13_slot_bytes,
                                         const void* codes2, int64_t codes2_slot_bytes,
                                         const void* scales2, int64_t scales2_slot_bytes,
                                         const void* zeros2, int64_t zeros2_slot_bytes,
                                         int scale_bf16, float routed_scaling_factor, void* y,
                                         unsigned int* err, void* stream);

/*
 * Loader relayout, bit-exact: uint8 [E, N, K/4] (value k at bits 2*(k%4) of byte k/4) ->
 * int32 [E, K/16, N]. Replaces to_word_ncontig() — gemv/moe_gemv_int2_tab.py:100-109, applied in
 * process_weights_after_loading (patches/ncontig_gemv.py:169-204).
 */
int w2a16_to_word_ncontig(const void* src_u8, void* dst_i32, int E, int N, int K, void* stream);

/*
 * Row gather through an address table: out[i, :] = the row_bytes bytes at tab[ids[i]].
 * Replaces _gather_rows_tab_kernel — patches/placement.py:34-43 (arena fill,
 * gemv/expert_elastic.py:45-51). row_bytes % 16 == 0, addresses 16-byte aligned.
 */
int w2a16_gather_rows_tab(const int64_t* tab, const int32_t* ids, int n, void* out, int64_t row_bytes,
                          void* stream);

/*
 * INT8 dense projection GEMV: y[m, n] = sum_k (q[k, n] - zero) * s[k / group, n] * x[m, k].
 * q packed 4 per int32 along K, int32 [K/4, N] (the auto_gptq layout of scripts/requant_int8.py:32-50);
 * scales f16 [K/group, N] (group == K: one scale per output channel). Replaces the GPTQ Marlin INT8
 * call SGLang makes for the dense projections (third party; docs/DECODE_PERF_PLAN.md:29).
 * x bf16 [M, K] (row stride stride_xm), y bf16 [M, N] (row stride stride_ym).
 * K % 128 == 0, N % 4 == 0, group % 128 == 0 and K % group == 0. Decode shapes (K <= 4096, M <= 8, N % 8 == 0,
 * scales 16-byte aligned) run one CTA per 32 output columns over all of K; other shapes reduce K slices inside
 * a thread-block cluster. Both are deterministic.
 */
int w2a16_int8_gemv(const void* x, int64_t stride_xm, const int32_t* qweight, const void* scales,
                    int group, int zero, int M, int K, int N, void* y, int64_t stride_ym,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes w2a16_int8_gemv accepts (a token amount: neither kernel uses global scratch; the argument
 * stays for ABI stability). */
size_t w2a16_int8_workspace_bytes(int M, int K, int N);

/* One-shot all-reduce (sum) of a small bf16 vector across the GPUs of one node over NVLink peer memory:
 * out[i] = sum over ranks r = 0..world-1 (in that order, fp32) of in_r[i], identical on every rank. Replaces
 * the per-layer NCCL all-reduce of the expert-parallel decode step (no counterpart in the reference, which
 * runs on one GPU). peer_bufs: device array of the `world` peer-visible buffer addresses (rank r's buffer
 * mapped into this process), each holding 2 x world x n_max bf16 and, at flag_offset bytes (>= 4 world n_max,
 * 16-byte multiple), `world` uint32 flags that are zero before the first call. epoch: this rank's device call
 * counter (zero initially). Every rank must make the same sequence of calls; n <= n_max, both multiples of 8,
 * `in` 16-byte aligned. A rank waits for every other rank's flag for at most spin_limit polls (0: the
 * library's default of 2^22, well above any healthy delay); a wait that gives up sets bit 1 of `err`, and the
 * call then completes with whatever rows are in place, so a lost rank is reported instead of hanging the GPU. */
int w2a16_allreduce_peers_bf16(const void* in, void* out, int n, int n_max, const uint64_t* peer_bufs,
                               size_t flag_offset, int rank, int world, unsigned int* epoch, unsigned int* err,
                               unsigned int spin_limit, void* stream);

/*
 * Exchange channel of an expert-parallel step. Each rank's peer-visible buffer holds, at tag_offset bytes (a
 * multiple of 16), 2 parity slots x world rows x n_max / 2 tagged 8-byte words: word j of row r carries values 2j
 * and 2j + 1 (bf16, low 32 bits) of rank r's partial of a call with that parity and the call number (high 32
 * bits), written and read as one single-copy-atomic access, so a reader polls the words it needs until they hold
 * its call -- no fences, counters or flags. Call e uses parity slot e & 1; epoch (device word, zero at the start)
 * counts the channel's calls on this rank. The same buffer and epoch word may serve w2a16_allreduce_peers_bf16
 * (its bf16 slots and flags below tag_offset), so a step can mix the calls.
 */
typedef struct w2a16_exchange {
  const uint64_t* peer_bufs;   /* device array [world] of the peer buffer addresses */
  size_t tag_offset;
  int n_max, rank, world;
  unsigned int* epoch;
  unsigned int spin_limit;     /* polls of a word before a wait gives up (bit 1 of err); 0 = library default */
} w2a16_exchange;

/* The slot-form decode layer of one expert-parallel rank with the exchange folded in (M * H <= n_max, one
 * per-token launch; no counterpart in the reference, which runs on one GPU). x_from_peers: x is not read; the
 * layer's activation is the sum, in rank order (fp32, rounded to bf16), of the ranks' rows of the channel's call
 * e = *epoch -- the all-reduce of the previous layer's partials, each word taken once it holds call e.
 * y_to_peers: y is not written; the layer's partial goes out as this rank's tagged row of call e + 1 into every
 * rank's buffer as its 32-column units finish, and *epoch becomes e + 1. With both, one launch per layer replaces
 * (layer, all-reduce). Other arguments as w2a16_moe_decode_layer_slots. */
int w2a16_moe_decode_layer_slots_ep(const void* x, int M, int H, int I, int top_k,
                                    const int32_t* topk_ids, const float* topk_w,
                                    const int32_t* slots, int num_experts, int num_slots,
                                    const void* codes13, int64_t codes13_slot_bytes,
                                    const void* scales13, int64_t scales13_slot_bytes,
                                    const void* zeros13, int64_t zeros13_slot_bytes,
                                    const void* codes2, int64_t codes2_slot_bytes,
                                    const void* scales2, int64_t scales2_slot_bytes,
                                    const void* zeros2, int64_t zeros2_slot_bytes,
                                    int scale_bf16, float routed_scaling_factor,
                                    void* y, void* workspace, size_t workspace_bytes,
                                    int x_from_peers, int y_to_peers, const w2a16_exchange* exchange,
                                    unsigned int* err, void* stream);

/* w2a16_int8_gemv with x the sum of the ranks' tagged rows of the channel's call *epoch (rows of K values,
 * M * K <= n_max): the dense projection after a pushing layer. Every shape runs the cluster kernel, whose CTAs
 * each poll only their K slice of every rank's row. */
int w2a16_int8_gemv_from_peers(const w2a16_exchange* exchange, const int32_t* qweight, const void* scales, int group,
                               int zero, int M, int K, int N, void* y, int64_t stride_ym, unsigned int* err,
                               void* stream);

/*
 * Native row arena for expert residency. Replaces RowArena (gemv/row_arena.py:34-123) and the virtual-memory
 * plumbing it borrows from SGLang: virtual addresses for max_rows rows of row_bytes are reserved once, and a
 * prefix of them is backed by physical memory in chunks (the device granularity rounds chunk_bytes up; 0 picks
 * 4 MiB). Growing maps chunks after the backed prefix; shrinking unmaps every chunk that lies entirely beyond the
 * rows kept and returns it to the driver. Row addresses (base + i * row_bytes) never change, so slot or address
 * tables into the arena -- and CUDA graphs captured over kernels that read them -- stay valid across resizes; a
 * table entry must only name backed rows. Not thread-safe per arena; resizes happen on the host between steps
 * (synchronise before a shrink if kernels may still read the rows being released).
 */
typedef struct w2a16_arena w2a16_arena;
int w2a16_arena_create(int device, int64_t row_bytes, int64_t max_rows, int64_t chunk_bytes, w2a16_arena** out);
/* Back rows [0, n) (n clamped to max_rows); adds the bytes newly mapped to *mapped_bytes (may be NULL).
 * W2A16_ERR_MEMORY when the device has no memory for another chunk (the chunks mapped so far stay). */
int w2a16_arena_ensure_rows(w2a16_arena* arena, int64_t n, int64_t* mapped_bytes);
/* Keep rows [0, n) backed and release every chunk entirely beyond row n; the bytes freed in *freed_bytes. */
int w2a16_arena_shrink_rows(w2a16_arena* arena, int64_t n, int64_t* freed_bytes);
uint64_t w2a16_arena_base(const w2a16_arena* arena);
int64_t w2a16_arena_backed_rows(const w2a16_arena* arena);
int64_t w2a16_arena_chunk_bytes(const w2a16_arena* arena);
/* Unmap and release every chunk and free the reserved addresses. */
int w2a16_arena_destroy(w2a16_arena* arena);

/* The driver calls an arena makes (each returns 0 on success), so the arena's bookkeeping can be exercised
 * against a fake: granularity of device allocations, reserve / free a virtual range, create / release a physical
 * chunk, map a chunk at an address with read-write access for the device / unmap it. ctx is passed back. */
typedef struct w2a16_vmm_driver {
  void* ctx;
  int (*granularity)(void* ctx, int device, uint64_t* bytes);
  int (*reserve)(void* ctx, uint64_t bytes, uint64_t* base);
  int (*free_va)(void* ctx, uint64_t base, uint64_t bytes);
  int (*create)(void* ctx, int device, uint64_t bytes, uint64_t* handle);
  int (*release)(void* ctx, uint64_t handle);
  int (*map)(void* ctx, int device, uint64_t va, uint64_t bytes, uint64_t handle);
  int (*unmap)(void* ctx, uint64_t va, uint64_t bytes);
} w2a16_vmm_driver;
/* w2a16_arena_create over the given driver table (w2a16_arena_create uses the CUDA driver's). */
int w2a16_arena_create_with_driver(const w2a16_vmm_driver* driver, int device, int64_t row_bytes, int64_t max_rows,
                                   int64_t chunk_bytes, w2a16_arena** out);

#ifdef __cplusplus
}
#endif

#endif /* W2A16_MOE_H */
