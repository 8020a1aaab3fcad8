/*
 * exl3_b200.h -- C ABI of the B200-native EXL3 routed-expert path.
 *
 * Every entry takes raw device pointers, element counts and a cudaStream_t
 * (passed as void*), and returns an int status (EXL3_OK or an EXL3_ERR_*
 * code); the message of the last failure on the calling thread is returned
 * by exl3_last_error().  Arguments are validated on the host before anything
 * is launched.  Kernels never trap: device-side problems (a null or
 * misaligned pointer inside a pointer table, a per-expert K outside 2..8, an
 * expired wait) record a code in the workspace's status word, read with
 * exl3_device_status().  No entry synchronises the stream and no entry
 * allocates device memory except where stated; work buffers are
 * caller-owned workspaces sized by the matching *_workspace_size query.
 *
 * Packed EXL3 tensor (reference: vcruz305/vllm-exl3
 * src/vllm_exl3/exl3.py:4405-4481, :113-117): trellis int16
 * [in/16][out/16][16*K], suh fp16 [in], svh fp16 [out]; codebook
 * 0 = 3INST, 1 = MCG, 2 = mul1.  in and out are multiples of 128.
 *
 * dtype codes: 0 = fp32, 1 = fp16, 2 = bf16, 3 = int32, 4 = int64.
 */
#ifndef EXL3_B200_H
#define EXL3_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EXL3_B200_ABI_VERSION 1

enum {
    EXL3_OK = 0,
    EXL3_ERR_ARG = 1,       /* invalid argument, rejected before launch */
    EXL3_ERR_CUDA = 2,      /* CUDA runtime error at launch */
    EXL3_ERR_WORKSPACE = 3  /* workspace missing or too small */
};

enum { EXL3_DT_F32 = 0, EXL3_DT_F16 = 1, EXL3_DT_BF16 = 2, EXL3_DT_I32 = 3, EXL3_DT_I64 = 4 };
enum { EXL3_CB_3INST = 0, EXL3_CB_MCG = 1, EXL3_CB_MUL1 = 2 };
/* MoE activations (src/vllm_exl3/exl3.py:143-154): SiLU-gated; non-gated relu^2
 * (no gate projection: the gate tables are not read); clamped SwiGLU-OAI. */
enum { EXL3_ACT_SILU = 0, EXL3_ACT_RELU2 = 2, EXL3_ACT_SWIGLU_OAI = 3 };

int exl3_abi_version(void);
const char* exl3_last_error(void);

/* Device status word of a workspace (0 = clean); `clear` resets it.  Reads
 * device memory synchronously on `stream`. */
int exl3_device_status(const void* workspace, int clear, void* stream, int* status_out);

/* Replaces dequant_trellis (csrc/bindings.cpp:117-132, CPU dequant_cpu
 * :15-100): W = diag(suh) H W~ H diag(svh) / 128 as fp16 [in][out],
 * bit-identical to the reference's CPU result.  K in 2..8. */
int exl3_reconstruct(const void* trellis, const void* suh, const void* svh, int64_t in_features,
                     int64_t out_features, int K, int codebook, void* w_out, void* stream);

/* Replaces ExLlamaV3 `reconstruct` (call sites src/vllm_exl3/exl3.py:3130-3156):
 * the decoded W~ as fp16 [in][out], no rotation. */
int exl3_decode_raw(const void* trellis, int64_t in_features, int64_t out_features, int K,
                    int codebook, void* w_out, void* stream);

/* Replaces ExLlamaV3 `had_r_128` (call sites src/vllm_exl3/exl3.py:3039-3156):
 * y = fp16(H128(x o pre) / sqrt(128) o post * scale) per 128-column block of
 * fp16 rows; pre and post may be NULL; y may alias x. */
int exl3_had128(const void* x, void* y, int64_t rows, int64_t n, const void* pre, const void* post,
                float scale, void* stream);

/* Replaces exl3_gemv (csrc/bindings.cpp:134-147, csrc/exl3_gemv.cu:23-63) and
 * exl3_gemm (csrc/exl3_gemm.cu:9-31): y[m][out] = x[m][in] W for any m.
 * x fp16/bf16/fp32 (cast to fp16 as the reference does), y in y_dtype. */
size_t exl3_linear_workspace_size(int64_t m, int64_t in_features, int64_t out_features, int K);
int exl3_linear(const void* x, int x_dtype, int64_t m, const void* trellis, const void* suh,
                const void* svh, int64_t in_features, int64_t out_features, int K, int codebook,
                void* y, int y_dtype, void* workspace, size_t workspace_bytes, void* stream);

/* Replaces p2b_fused_moe / p2b_fused_moe_mk / p2b_fused_moe_padded
 * (csrc/bindings.cpp:158-241, csrc/p2b_moe.cu:643-2428) and ExLlamaV3
 * exl3_moe / exl3_moe_mixedk (call sites src/vllm_exl3/exl3.py:3495-3579):
 * the routed-expert layer for ALL tokens in one call,
 *   out[t] = sum_k w[t][k] * down_e(act(gate_e(x[t]), up_e(x[t]))),  e = local(ids[t][k]).
 * Pointer tables: nine int64 device arrays [n_table] of per-expert data
 * pointers, the layout of build_exl3_fused_state (exl3.py:2475-2508).
 * K: per-expert int8 device tables k_gate/k_up/k_down [n_table] (mixed-K,
 * p2b_fused_moe_mk) or, when they are NULL, the uniform k_uniform.
 * ids [tokens][topk] int32/int64 global expert ids; expert_map (int32
 * [n_global], may be NULL) maps them to local ids (exl3.py:2332-2354); ids
 * that are negative, out of range or map outside [0, n_local) are skipped.
 * n_valid (int32[1] device, may be NULL) limits live tokens; rows at or past
 * it are written as zeros (p2b_fused_moe_padded).  swiglu_limit > 0 clamps
 * gate from above and up on both sides (p2b_moe.cu:755-768).  activation:
 * EXL3_ACT_SILU silu(g) * u; EXL3_ACT_SWIGLU_OAI (u + 1) g sigmoid(1.702 g);
 * EXL3_ACT_RELU2 relu(u)^2 for non-gated layers (exl3.py:2386-2391), whose
 * gate tables may alias the up tables and are never read.  out [tokens][hidden]
 * in out_dtype.  `kmax` bounds every K in the tables (2..8). */
size_t exl3_moe_workspace_size(int64_t tokens, int topk, int64_t hidden, int64_t intermediate,
                               int n_local, int kmax);
int exl3_moe_forward(const void* x, int x_dtype, int64_t tokens, int64_t hidden,
                     int64_t intermediate, const int64_t* gate_trellis_ptrs,
                     const int64_t* gate_suh_ptrs, const int64_t* gate_svh_ptrs,
                     const int64_t* up_trellis_ptrs, const int64_t* up_suh_ptrs,
                     const int64_t* up_svh_ptrs, const int64_t* down_trellis_ptrs,
                     const int64_t* down_suh_ptrs, const int64_t* down_svh_ptrs,
                     const void* topk_ids, int ids_dtype, const void* topk_weights, int w_dtype,
                     int topk, const int32_t* expert_map, int64_t n_global, const int8_t* k_gate,
                     const int8_t* k_up, const int8_t* k_down, int k_uniform, int kmax,
                     int n_local, int codebook, int activation, float swiglu_limit,
                     const int32_t* n_valid, void* out, int out_dtype, void* workspace,
                     size_t workspace_bytes, void* stream);

/* Replaces p2b_gemv_batched (csrc/bindings.cpp:149-156, csrc/p2b_batched.cu:341-368):
 * one shared input x [m][in] against the experts listed in expert_indices
 * (int32 device [n_active], entries indexing the tables [n_table]);
 * y [n_active][m][out] with y[j] = x W_{expert_indices[j]}.  Entries outside
 * [0, n_table) leave their rows untouched.  The reference fixes out = 2048
 * and K in 2..4; here out is any multiple of 128 and K is 2..8. */
size_t exl3_batched_linear_workspace_size(int64_t m, int n_active, int64_t in_features,
                                          int64_t out_features, int n_table, int K);
int exl3_batched_linear(const void* x, int x_dtype, int64_t m, const int64_t* trellis_ptrs,
                        const int64_t* suh_ptrs, const int64_t* svh_ptrs, int n_table,
                        const int32_t* expert_indices, int n_active, int64_t in_features,
                        int64_t out_features, int K, int codebook, void* y, int y_dtype,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Replaces exl3_fat_gemm / exl3_fat_gemm_scatter (csrc/exl3_fat_gemm.cu:266-305):
 * `a` fp16 [m][in] is already input-rotated (had_r_128 of the activations
 * with suh); out fp32 = (a W~) H / sqrt(128) o svh.  Without token_idx it
 * writes out [m][out]; with token_idx (int64 [m]) and route_weight (fp16 [m])
 * it adds route_weight[r] * row r into out[token_idx[r]] -- a plain
 * read-modify-write, race-free only when no two rows of one call share a
 * token, the reference's contract (exl3_fat_gemm.cu:182-189).  Any K 2..8
 * and codebook (the reference: K4 MCG only).  Workspace: exl3_linear_workspace_size. */
int exl3_fat_gemm(const void* a, int64_t m, const void* packed, const void* svh, int64_t in_features,
                  int64_t out_features, int K, int codebook, float* out, const int64_t* token_idx,
                  const void* route_weight, void* workspace, size_t workspace_bytes, void* stream);

/* exl3_linear for callers that cannot allocate device memory when they run
 * a projection (no counterpart in the reference): e.g. a serving engine that
 * has already given all free HBM to its KV cache, or a C/FFI host with no
 * caching allocator, where every cudaMalloc/cudaFree would also synchronise.
 * Same arguments and result as exl3_linear minus the workspace: the work
 * buffers live in one file-scope device array of
 * EXL3_LINEAR_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds
 * until exit.  Calls needing more scratch are rejected (EXL3_ERR_ARG) before
 * anything is launched.  The first call on a device looks up the array's
 * address with that device current; make it before any stream capture.
 * All calls share the array: calls whose GPU work overlaps race.  The call
 * itself allocates nothing (no cudaMalloc, cudaFree or allocating library). */
#define EXL3_LINEAR_NOALLOC_SCRATCH_BYTES (16u << 20)
int exl3_linear_noalloc(const void* x, int x_dtype, int64_t m, const void* trellis, const void* suh,
                        const void* svh, int64_t in_features, int64_t out_features, int K,
                        int codebook, void* y, int y_dtype, void* stream);

/* Row-wise EXL3 embedding tables in the n-gram format (replaces ExLlamaV3's
 * ngram_dequant, call site src/vllm_exl3/exl3.py:5536-5544, restated by the
 * reference as ngram_dequant_rows_torch, exl3.py:5213-5239).  A row of `bits`
 * (1..8) is 1 + 10 * bits int16 words: an fp16 scale, then a ring bitstream of
 * 160 states; out[r][i] = fp16(mul1(state_i) * scale + head_bias[head][i]),
 * written in out_dtype.  exl3_ngram_dequant decodes `n` packed rows with a
 * head index each (int32 [n], clamped to [0, num_heads)).  exl3_ngram_lookup
 * is the whole lookup of Exl3EmbeddingMethod._embedding_impl (exl3.py:
 * 5576-5587) in one launch: row ids [n] (int32/int64) gathered from a table
 * of n_rows rows, each id's head = (number of head_offsets <= id) - 1
 * clamped (searchsorted, right), then decoded; ids outside the table give
 * zero rows and record status 7 in `status` (an int32 device word, may be
 * NULL).  head_bias fp16 [num_heads][160]. */
int exl3_ngram_dequant(const void* packed, int64_t n, int bits, const int32_t* heads, const void* head_bias,
                       int num_heads, void* out, int out_dtype, void* stream);
int exl3_ngram_lookup(const void* table, int64_t n_rows, int bits, const void* ids, int ids_dtype, int64_t n,
                      const int64_t* head_offsets, int num_heads, const void* head_bias, void* out, int out_dtype,
                      int* status, void* stream);

/* Expert-parallel dispatch, source side (no counterpart in the reference,
 * which leaves the exchange to vLLM's all-to-all backends and consumes only
 * the resulting expert_map, src/vllm_exl3/exl3.py:2310-2354).  Rank g of
 * `world` owns global experts [g*E/world, (g+1)*E/world), E = n_global
 * (a multiple of world).  A host with another expert placement maps each
 * global id to its slot in that order before the call.  For every token
 * t < n_valid (all tokens when
 * n_valid is NULL) and every rank g owning at least one of its routes it
 * writes one pair p: send_x[p] = x[t], send_ids[p][k] = the local id of
 * route k on g or -1, send_w[p][k] = its weight (fp32) or 0, send_tok[p] = t,
 * pair_idx[t][g] = p (-1 where t sends nothing to g).  Pairs are rank-major
 * and token-ascending inside a rank; send_counts[g] = rank g's pairs, so rank
 * g's rows are the contiguous block after the counts of ranks < g.  Size the
 * pair buffers for tokens * min(world, topk) rows.  With capacity C > 0
 * (C >= tokens, the same on every rank) rank g's pairs instead fill rows
 * [g*C, g*C + send_counts[g]) of fixed C-row blocks; the other slots get
 * send_tok -1, ids -1 and weight 0 (their send_x rows are not written), so
 * the exchange is an equal-split all-to-all of C rows per rank and no count
 * has to reach the host; size the buffers for world * C rows.  Routes with
 * ids outside [0, E) are dropped.  x fp32/fp16/bf16 [tokens][hidden], hidden
 * a multiple of 128, x and send_x 16-byte aligned. */
int exl3_ep_dispatch(const void* x, int x_dtype, int64_t tokens, int64_t hidden, const void* topk_ids,
                     int ids_dtype, const void* topk_weights, int w_dtype, int topk, int64_t n_global,
                     int world, const int32_t* n_valid, void* send_x, int32_t* send_ids, float* send_w,
                     int32_t* send_tok, int32_t* pair_idx, int32_t* send_counts, int64_t capacity,
                     void* stream);

/* Expert-parallel combine, source side (no reference counterpart; see
 * exl3_ep_dispatch): out[t] = sum over ranks g = 0, 1, ... of
 * partial[pair_idx[t][g]] where that is >= 0, accumulated in fp32 in that
 * fixed order (deterministic, no atomics); rows t >= n_valid are zero.
 * partial fp32/fp16/bf16 [pairs][hidden], out fp32/fp16/bf16 [tokens][hidden],
 * both 16-byte aligned. */
int exl3_ep_combine(const void* partial, int partial_dtype, const int32_t* pair_idx, int64_t tokens, int world,
                    int64_t hidden, const int32_t* n_valid, void* out, int out_dtype, void* stream);

/* Expert-parallel exchange over NVLink peer memory (no counterpart in the
 * reference; replaces the NCCL all-to-all around exl3_ep_dispatch /
 * exl3_ep_combine with direct stores into the peers' memory).
 *
 * Every rank allocates a window of exl3_ep_window_size bytes (the same
 * geometry on all ranks: world, capacity rows per rank pair, hidden, topk,
 * the dtypes of the token rows and of the partial rows), exports it with
 * exl3_ep_ipc_handle and maps its peers' windows with exl3_ep_ipc_open;
 * `peers` is a device int64 array of `world` window addresses as seen from
 * this GPU (its own entry = its own window).  A layer step on every rank:
 *   exl3_ep_p2p_dispatch  pair the tokens with their owners (as
 *                         exl3_ep_dispatch with a capacity) and store each
 *                         pair's row, local ids and weights into its owner's
 *                         window, then raise this step's arrival flag there;
 *   exl3_ep_p2p_wait(0)   wait until every peer's rows have arrived;
 *   exl3_moe_forward      on the window's received rows (world * capacity
 *                         rows at exl3_ep_window_recv, ids -1 marking empty
 *                         slots) into a partial buffer;
 *   exl3_ep_p2p_return    store each source's partial rows back into its
 *                         window and raise the return flag there;
 *   exl3_ep_p2p_wait(1)   wait until every owner's partial rows are back;
 *   exl3_ep_p2p_combine   per-token sum over owners in rank order (as
 *                         exl3_ep_combine), then advance the step counter.
 * Flags carry the step number, so nothing is reset between steps and the
 * whole step can be captured in a CUDA graph; a step completes the round
 * trip before the next begins, so each direction needs one buffer.  Waits
 * are bounded (about 2 s): a timeout records status 4 in the window's
 * status word (read it with exl3_device_status(window + 4)) instead of
 * hanging.  Allocation and IPC calls are synchronous; make them before any
 * stream capture. */
size_t exl3_ep_window_size(int world, int64_t capacity, int64_t hidden, int topk, int x_dtype, int partial_dtype);
int exl3_ep_window_alloc(size_t bytes, void** window);
int exl3_ep_window_free(void* window);
int exl3_ep_ipc_handle(const void* window, void* handle /* 64 bytes */);
int exl3_ep_ipc_open(const void* handle, void** mapped);
int exl3_ep_ipc_close(void* mapped);
int exl3_ep_p2p_dispatch(const void* x, int x_dtype, int64_t tokens, int64_t hidden, const void* topk_ids,
                         int ids_dtype, const void* topk_weights, int w_dtype, int topk, int64_t n_global,
                         int world, int rank, int64_t capacity, const int32_t* n_valid, void* window,
                         const int64_t* peers, int partial_dtype, int32_t* pair_idx, void* stream);
int exl3_ep_p2p_wait(void* window, int world, int phase, void* stream);
int exl3_ep_p2p_return(const void* partial, int partial_dtype, int world, int rank, int64_t capacity,
                       int64_t hidden, int topk, int x_dtype, void* window, const int64_t* peers, void* stream);
int exl3_ep_p2p_combine(void* window, int world, int rank, int64_t capacity, int64_t hidden, int topk,
                        int x_dtype, int partial_dtype, const int32_t* pair_idx, int64_t tokens,
                        const int32_t* n_valid, void* out, int out_dtype, void* stream);
/* Byte offsets of the received rows, local ids (int32) and weights (fp32)
 * inside a window of that geometry (what exl3_moe_forward reads). */
int exl3_ep_window_recv(int world, int64_t capacity, int64_t hidden, int topk, int x_dtype, int partial_dtype,
                        size_t* x_off, size_t* ids_off, size_t* w_off);

/* Phase timing for benchmarks (no reference counterpart; the reference times
 * its kernels with CUDA events in tools/bench_moe_decode.py:24-55).  While
 * enabled, exl3_moe_forward and exl3_linear first launch a spin of
 * `delay_cycles` GPU clocks (capped at 4e9) so every launch is queued before
 * the GPU reaches it, then record a CUDA event before and after each kernel
 * phase on the call's stream: MoE = prep, rotate, gate/up, down, combine;
 * linear = prep, rotate, gemv.  exl3_profile_read waits for the last call's
 * final event and returns each phase's milliseconds.  Process-global, not
 * thread-safe, not for use inside CUDA-graph capture. */
int exl3_profile_enable(int on, long long delay_cycles);
int exl3_profile_read(float* ms, int max_phases, int* n_phases);

#ifdef __cplusplus
}
#endif

#endif /* EXL3_B200_H */
