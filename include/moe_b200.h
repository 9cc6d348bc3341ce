/*
 * moe_b200.h - C ABI of the B200 (sm_100a) MoE expert-layer forward path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t,
 * launches asynchronously on that stream and returns a moe_status. On a
 * non-zero status, moe_b200_last_error() returns a message for the calling
 * thread. Outputs are caller-allocated; inputs are only read. No entry point
 * synchronises the stream or allocates device memory (moe_grouped_gemm_check
 * and moe_permute_check, which read a device error word back to the host,
 * are the calls that wait); the ones that need scratch take a caller-provided
 * workspace whose size the matching *_workspace_size function reports.
 *
 * Each function names the reference interface it replaces. The reference
 * binds its kernels through pybind functions that take torch tensors and call
 * a raw-pointer launcher on the default stream; this header is the raw-pointer
 * layer, with an explicit stream and a status code added.
 *
 * Row-id maps follow the reference convention: entry >= 0 is a destination
 * (permute) or source (unpermute) row of the expert-major permuted buffer,
 * -1 means "token not routed to this expert".
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* moe_stream_t; /* == cudaStream_t */

typedef enum {
  MOE_OK = 0,
  MOE_ERR_INVALID = 1,     /* bad argument: null pointer, size, alignment, dtype code */
  MOE_ERR_UNSUPPORTED = 2, /* valid but outside what this build supports (e.g. k > 16) */
  MOE_ERR_CUDA = 3,        /* a CUDA runtime/driver call or launch failed */
  MOE_ERR_DEVICE = 4       /* a kernel reported an error word (see moe_grouped_gemm) */
} moe_status;

/* Message for the last failing call on this host thread ("" if none). */
const char* moe_b200_last_error(void);
/* ABI version: bumped on any signature change. */
int moe_b200_abi_version(void);

/* ------------------------------------------------------------------------ */
/* a1  Row-wise top-k, largest, sorted, ties -> lower column index.          */
/* Replaces kernel_results/case23_aten_topk/binding.cpp:4 (launch_topk) and  */
/* matches kernel_cases/case23_ref_aten_topk.py:47-62 (reference_topk).      */
/* input [M,N] fp32 row-major; values [M,k] fp32; indices [M,k] int64.       */
/* 1 <= k <= min(N, 16) and N <= 2048, else MOE_ERR_UNSUPPORTED. NaN ranks   */
/* first, as in torch.sort / torch.topk.                                     */
int moe_topk_f32(const float* input, float* values, int64_t* indices, int64_t M, int64_t N,
                 int32_t k, moe_stream_t stream);

/* a1+a2  Fused router: score -> top-k -> gate weights -> routing map.       */
/* score_mode 0: select on the raw logits, gate = logit.                     */
/* score_mode 1: softmax over the row, gate = softmax prob; with renorm != 0 */
/*               the k selected probs are rescaled to sum to 1.              */
/* Selection order is the logits' (softmax is monotone); ties -> lower index.*/
/* bias (nullable, [E] fp32) is added to the logits before everything.       */
/* Outputs (each nullable): topk_vals [T,k] fp32, topk_idx [T,k] int64,      */
/* routing_map [T,E] uint8/bool, probs [T,E] fp32 (gate at selected, else 0).*/
/* The routing map and dense probs are the inputs the reference builds with  */
/* scatter_ (kernel_cases/case12_moe_row_id_map_pass2.py:30-40,              */
/* kernel_cases/case17_moe_permute_with_mask_map.py:78-90).                  */
int moe_router_topk(const float* logits, const float* bias, int64_t T, int64_t E, int32_t k,
                    int32_t score_mode, int32_t renorm, float* topk_vals, int64_t* topk_idx,
                    uint8_t* routing_map, float* probs, moe_stream_t stream);

/* Router over a placement of the experts: slot c of every output (routing  */
/* map, probs and topk_idx columns) is model expert placement[c] (an int32   */
/* permutation of [0,E) on the device), so experts placed on one GPU get     */
/* contiguous slots and contiguous permuted rows. Ties rank the lower slot   */
/* first. Same arithmetic as moe_router_topk otherwise.                      */
int moe_router_topk_placed(const float* logits, const float* bias, const int32_t* placement,
                           int64_t T, int64_t E, int32_t k, int32_t score_mode, int32_t renorm,
                           float* topk_vals, int64_t* topk_idx, uint8_t* routing_map,
                           float* probs, moe_stream_t stream);

/* f1  Router gate GEMM fused with the router above, one kernel:             */
/*   logits = x @ w^T (x [T,H] bf16, w [E,H] bf16, fp32 accumulation on the */
/*   tensor cores), then exactly moe_router_topk on those logits (same       */
/*   selection, gate formula and summation order, so the same bits).         */
/* Replaces kernel_cases/case38_ref_musa_asm_bf16_ssgemm_nt_320x256.py:51-59 */
/* (the router gate GEMM) followed by moe_router_topk, without the [T,E]     */
/* fp32 logits round trip through HBM.                                       */
/* H % 8 == 0; E a multiple of 32 in [32, 512]; 1 <= k <= min(E, 16).        */
/* Outputs are nullable: logits [T,E] fp32 (the unbiased GEMM result),       */
/* topk_vals/topk_idx [T,k], routing_map [T,E] uint8, probs [T,E] fp32.      */
/* With only logits requested this is the plain router GEMM. x, w, logits,   */
/* routing_map and probs must be 16-byte aligned.                            */
/* device_error: device int32, zero before the first call; a kernel whose    */
/* bounded wait expired stores a nonzero code there (never cleared here).    */
int moe_router_gemm_topk(const void* x, const void* w, const float* bias, int64_t T, int64_t H,
                         int64_t E, int32_t k, int32_t score_mode, int32_t renorm, float* logits,
                         float* topk_vals, int64_t* topk_idx, uint8_t* routing_map, float* probs,
                         int32_t* device_error, moe_stream_t stream);

/* ------------------------------------------------------------------------ */
/* a3  routing_map [T,E] bool -> row_id_map, expert-major destinations:      */
/*   row[t,e] = base[e] + #{t' <= t : map[t',e]} - 1 if map[t,e] else -1     */
/* base[e] = sum over e' < e of roundup(count[e'], align) (align = 1 is the  */
/* reference's make_row_id_map, kernel_cases/case12_moe_row_id_map_pass2.py: */
/* 43-50; larger aligns pad every expert segment for tile-aligned GEMMs).    */
/* Replaces the five launchers of kernel_results/case12_moe_row_id_map_pass2 */
/* /binding.cpp:7-11. Outputs (nullable except one of the maps):             */
/*   row_id_map_et [E,T] int64, row_id_map_te [T,E] int64,                   */
/*   expert_counts [E] int32, num_out [1] int64 (padded total rows).          */
int moe_row_id_map_workspace_size(int64_t T, int64_t E, size_t* bytes);
int moe_row_id_map(const uint8_t* routing_map, int64_t T, int64_t E, int64_t align,
                   int64_t* row_id_map_et, int64_t* row_id_map_te, int32_t* expert_counts,
                   int64_t* num_out, void* workspace, size_t workspace_bytes,
                   moe_stream_t stream);

/* Same maps as moe_row_id_map, for callers that may not allocate device     */
/* memory (a runtime that owns a fixed HBM budget, or a path where          */
/* cudaMalloc's implicit synchronisation is not allowed). No counterpart in  */
/* the reference. Its scratch is a 1 MiB file-scope device array held by     */
/* every GPU that loads the library. A call needs                           */
/*   roundup(E * ceil(T/64) * 4, 256) + roundup(E * 8, 256) <= 1 MiB         */
/* bytes of it (at E=256: T <= 65408); larger sizes are rejected with        */
/* MOE_ERR_INVALID before any device work. The first call on a device looks  */
/* the array's address up and caches it for the life of the process (make   */
/* that call before any stream capture, and do not use the library across a */
/* cudaDeviceReset of that device). Calls share the array: calls that        */
/* overlap on the GPU race.                                                  */
int moe_row_id_map_static_scratch(const uint8_t* routing_map, int64_t T, int64_t E,
                                  int64_t align, int64_t* row_id_map_et, int64_t* row_id_map_te,
                                  int32_t* expert_counts, int64_t* num_out, moe_stream_t stream);

/* ------------------------------------------------------------------------ */
/* a4  Permute with a [T,E] map: out[row[t,e]] = x[t], pp[row[t,e]] =        */
/* probs[t,e]. Replaces kernel_results/case17_moe_permute_with_mask_map/     */
/* binding.cpp:5-6 (permute_rt_launcher); semantics of kernel_cases/case17_  */
/* moe_permute_with_mask_map.py:58-71. x/out bf16 (any 2-byte type: pure     */
/* copy), any H; rows move as 16-, 4- or 2-byte vectors depending on H and   */
/* pointer alignment. probs / permuted_probs nullable together. Rows of out  */
/* no map entry points at are left untouched; entries outside [0, num_out)   */
/* are skipped.                                                              */
int moe_permute_mask_map(const void* x, const int64_t* row_id_map_te, const float* probs,
                         void* out, float* permuted_probs, int64_t T, int64_t H, int64_t E,
                         int64_t num_out, moe_stream_t stream);

/* a4  Same permute driven by the router's expert list topk_experts [T,k]    */
/* int64 (k <= 32, any order): the destination of (t, j) is                  */
/* map[t, topk_experts[t,j]], so the kernel reads k map entries per token    */
/* instead of the whole E-entry row. Same output as moe_permute_mask_map;    */
/* 16-byte rows (H % 8 == 0, aligned pointers), H <= 8192.                   */
int moe_permute_topk(const void* x, const int64_t* row_id_map_te, const int64_t* topk_experts,
                     int32_t k, const float* probs, void* out, float* permuted_probs, int64_t T,
                     int64_t H, int64_t E, int64_t num_out, moe_stream_t stream);

/* a5  Same with an expert-major [E,T] map of int64 (idx_bits 64) or int32   */
/* (idx_bits 32): kernel_cases/case22_ref_moe_permute_mask_kernel_true.py:   */
/* 47-69, case21_ref_permute_with_mask_map_trans.py:52-68,                   */
/* case30_ref_moe_permute_mask_kernel.py:44-58 (probs null).                 */
int moe_permute_mask_map_trans(const void* x, const void* row_id_map_et, int32_t idx_bits,
                               const float* probs, void* out, float* permuted_probs, int64_t T,
                               int64_t H, int64_t E, int64_t num_out, moe_stream_t stream);

/* With MOE_PERMUTE_BULK=1 in the environment, rows with 16-byte aligned     */
/* pointers and H <= 16384 (H % 8 == 0) go through the bulk-copy (TMA)        */
/* engine instead of registers: one bulk load of each token row into shared   */
/* memory, one bulk store per destination row. Its bounded wait on a row      */
/* load records a device error word; moe_permute_check reads it back (and     */
/* clears it), synchronising `stream`: 0 = none, 1 = a row load timed out.    */
/* No reference counterpart (the reference launchers return nothing).         */
int moe_permute_check(moe_stream_t stream, int32_t* device_error);

/* ------------------------------------------------------------------------ */
/* a6/a7/a8  Unpermute (combine) with an expert-major [E,T] map:             */
/*   acc[t] = sum over e ascending of w(t,e) * float(pin[row[e,t]])          */
/*   out[t] = bf16_rne(acc[t]); acc_out (nullable, [T,H] fp32) = acc.         */
/* w = 1 when probs is null (kernel_results/case15_moe_unpermute_mask_fwd/   */
/* binding.cpp:5-8, kernel_cases/case15_moe_unpermute_mask_fwd.py:58-64,    */
/* case24_ref_moe_unpermute_mask_kernel_false.py:45-68); otherwise           */
/* w = probs[t,e] ([T,E] fp32, probs_mode 0) or w = probs[row[e,t]]          */
/* (permuted [num_rows] fp32, probs_mode 1). Products and sums are separate  */
/* fp32 roundings (no FMA), accumulated in ascending expert order.           */
/* Any H up to 16384 (16-byte rows), 4096 (4-byte) or 2048 (2-byte).         */
int moe_unpermute_mask(const void* pin, const void* row_id_map_et, int32_t idx_bits,
                       const float* probs, int32_t probs_mode, void* out, float* acc_out,
                       int64_t T, int64_t H, int64_t E, int64_t num_rows, moe_stream_t stream);

/* Backward of the permute (kernel_cases/case18_moe_permute_bwd_unpermute_   */
/* mask.py:56-70 with an int64 map, case32_ref_moe_unpermute_mask_kernel.py: */
/* 47-79 with an int32 map): grad_x[t] = bf16(sum over e ascending of        */
/* fp32(grad_permuted[map[e,t]])) (acc_out, optional, the fp32 sums), and    */
/* grad_probs[t,e] = permuted_probs_grad[map[e,t]] for a routed (t,e), else  */
/* 0 (both optional, together; [T,E] fp32).                                  */
int moe_permute_backward(const void* grad_permuted, const void* row_id_map_et, int32_t idx_bits,
                         const float* permuted_probs_grad, void* grad_x, float* acc_out,
                         float* grad_probs, int64_t T, int64_t H, int64_t E, int64_t num_rows,
                         moe_stream_t stream);

/* f3  Backward of the prob-weighted combine (the forward is                 */
/* moe_unpermute_mask_token_major with dense probs; no reference kernel,     */
/* the chain rule of out[t] = sum_e probs[t,e] * rows[map[t,e]]):            */
/*   grad_rows[map[t,e]] = bf16(probs[t,e] * grad_out[t])                    */
/*   grad_probs[t,e] = <grad_out[t], rows[map[t,e]]> in fp32, 0 if unrouted. */
/* grad_out [T,H] bf16, rows [num_rows,H] bf16 (the forward's fc2 output),   */
/* row_id_map_te [T,E] int64, probs [T,E] fp32; E <= 1024. Rows that no      */
/* token references are not written.                                         */
int moe_combine_backward(const void* grad_out, const void* rows, const int64_t* row_id_map_te,
                         const float* probs, void* grad_rows, float* grad_probs, int64_t T,
                         int64_t H, int64_t E, int64_t num_rows, moe_stream_t stream);

/* f3  Backward of SwiGLU (h = silu(g) * u, y = [g | u] per row):            */
/* dy = [dh * u * silu'(g) | dh * silu(g)] in fp32 from bf16 inputs, rounded */
/* to bf16. y [M,2F], dh [M,F], dy [M,2F] bf16, F % 8 == 0, 16-byte aligned. */
int moe_swiglu_backward(const void* y, const void* dh, void* dy, int64_t M, int64_t F,
                        moe_stream_t stream);

/* Same combine driven by the token-major [T,E] int64 map (the layout         */
/* kernel_cases/case12_moe_row_id_map_pass2.py:61 returns second), whose     */
/* entries for one token are contiguous. Identical results. E <= 1024.       */
int moe_unpermute_mask_token_major(const void* pin, const int64_t* row_id_map_te,
                                   const float* probs, int32_t probs_mode, void* out,
                                   float* acc_out, int64_t T, int64_t H, int64_t E,
                                   int64_t num_rows, moe_stream_t stream);

/* ------------------------------------------------------------------------ */
/* a9/a10/a11  Grouped GEMM on tcgen05 tensor cores (bf16 in, fp32 acc).     */
/* out[r, :] = x[r, :] @ w[widx(g)]^T for the rows r of group g, where       */
/* w is [num_w, N, K] ("[out,in]" as in kernel_cases/case03_moe_grouped_gemm */
/* _fc1_fwd.py:57-64 and case04_moe_grouped_gemm_fc2_fwd.py:57-64).          */
/* Groups are described on the device by a group table built with            */
/* moe_grouped_gemm_plan_* below, so no host synchronisation is needed.      */
/* epilogue 0: out [rows, N] bf16.                                           */
/* epilogue 1 (SwiGLU, fc1): N = 2F with rows [0,F) = gate, [F,2F) = up;     */
/*   out [rows, F] bf16 = silu(g) * u with g, u the bf16-rounded GEMM        */
/*   outputs (the unfused chain fc1 -> bf16 -> silu(gate)*up).               */
/* epilogue 2: out [rows, N] fp32, the accumulator unrounded. With G = 1     */
/*   this is the router logits GEMM logits = inp @ weight^T (bf16 in, fp32   */
/*   out), replacing kernel_cases/case38_ref_musa_asm_bf16_ssgemm_nt_320x256 */
/*   .py:51-59 (reference_fp32; the muDNN TN GEMM of the router gate).       */
/* x [x_rows, K] bf16, K % 8 == 0, N % 8 == 0 (F % 8 for SwiGLU).            */
/* workspace: moe_grouped_gemm_workspace_size(G) bytes, 256-byte aligned.    */
int moe_grouped_gemm_workspace_size(int64_t G, size_t* bytes);

/* Plan from per-group row counts (device int32 [G], contiguous groups in    */
/* order; each group's first row rounded up to `align`): widx(g) = g.        */
int moe_grouped_gemm_plan_splits(const int32_t* m_splits, int64_t G, int64_t align,
                                 void* workspace, size_t workspace_bytes, moe_stream_t stream);

/* Plan for expert-parallel receive buffers: rows arrive as num_src blocks   */
/* (one per source rank) of num_w expert segments each, counts[s*num_w + e]. */
/* Groups are ordered expert-major (all sources of expert 0, then expert 1), */
/* so each weight matrix is streamed once; widx(g) = e.                      */
int moe_grouped_gemm_plan_ep(const int32_t* counts, int64_t num_src, int64_t num_w,
                             void* workspace, size_t workspace_bytes, moe_stream_t stream);

int moe_grouped_gemm(const void* x, const void* w, void* out, int64_t x_rows, int64_t G,
                     int64_t num_w, int64_t N, int64_t K, int32_t epilogue,
                     const void* workspace, size_t workspace_bytes, moe_stream_t stream);

/* f3  Same with w [num_w, K, N] (N contiguous): out[r, :] = x[r, :] @        */
/* w[widx(g)] — the grouped dgrad dx = dy @ W of the forward weight as it is  */
/* (kernel_cases/case07_moe_grouped_gemm_fc1_dgrad.py:49-64,                 */
/* case08_moe_grouped_gemm_fc2_dgrad.py:49-64; case13/case19 with G = 1).    */
/* The weight tile is staged MN-major (no transposed copy). Epilogue 0 or 2. */
int moe_grouped_gemm_nn(const void* x, const void* w, void* out, int64_t x_rows, int64_t G,
                        int64_t num_w, int64_t N, int64_t K, int32_t epilogue,
                        const void* workspace, size_t workspace_bytes, moe_stream_t stream);

/* f3  Grouped weight gradient: dW[g] = dy[rows of g]^T @ x[rows of g],      */
/* dy [rows_total, N], x [rows_total, K] bf16 row-major, groups contiguous   */
/* in order with row counts m_splits[G] (sum <= rows_total), dW [G, N, K]    */
/* bf16 (fp32 accumulation); a group with no rows gets zeros.                */
/* Replaces the torch.mm(dy[seg].t(), x[seg]) loop of kernel_cases/case05_   */
/* moe_grouped_gemm_fc2_wgrad.py:49-64 and case09_moe_grouped_gemm_fc1_      */
/* wgrad.py:49-64 ("TN"). The group table and one pair of tensor maps per    */
/* group with rows are built on the device, in the workspace                 */
/* (moe_grouped_wgrad_workspace_size), from two host-encoded templates; its  */
/* first 4 bytes are the device error word (read it with                     */
/* moe_grouped_gemm_check; 4 = a negative count or sum(m_splits) beyond      */
/* rows_total, in which case only the empty groups are written).             */
/* moe_grouped_wgrad: m_splits is a host array, G <= 4096 (passed by value   */
/* in the launch, so nothing waits for the stream).                          */
/* moe_grouped_wgrad_dev: m_splits is a device array (e.g. the expert        */
/* counts of moe_row_id_map), G <= 2^20; the CTA-pair kernel is chosen when  */
/* rows_total / G >= 384.                                                    */
int moe_grouped_wgrad_workspace_size(int64_t G, size_t* bytes);
int moe_grouped_wgrad(const void* dy, const void* x, void* dw, int64_t rows_total, int64_t G,
                      int64_t N, int64_t K, const int32_t* m_splits, void* workspace,
                      size_t workspace_bytes, moe_stream_t stream);
int moe_grouped_wgrad_dev(const void* dy, const void* x, void* dw, int64_t rows_total,
                          int64_t G, int64_t N, int64_t K, const int32_t* m_splits,
                          void* workspace, size_t workspace_bytes, moe_stream_t stream);

/* Reads the device error word a previous moe_grouped_gemm left in the       */
/* workspace (0 = none; blocking: synchronises the stream).                  */
int moe_grouped_gemm_check(const void* workspace, size_t workspace_bytes, moe_stream_t stream,
                           int32_t* device_error);

/* a11 standalone: h[M,F] = bf16(silu(y[:, :F]) * y[:, F:]) for y [M,2F].    */
int moe_swiglu(const void* y, void* h, int64_t M, int64_t F, moe_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Expert-parallel exchange over NVLink (e): receive buffers registered for  */
/* peer access with CUDA IPC, rows pushed by the copy engines. Stands in for  */
/* the intranode deep_ep dispatch / combine the reference names but does not */
/* contain (kernel_cases/case22_ref_moe_permute_mask_kernel_true.py:3-6,     */
/* case24_ref_moe_unpermute_mask_kernel_false.py:3-6).                        */
/* handle: 64 bytes (cudaIpcMemHandle_t) of the allocation holding dev_ptr;  */
/* offset: dev_ptr minus that allocation's base.                             */
int moe_ipc_get_handle(const void* dev_ptr, void* handle_out, uint64_t* offset_out);
int moe_ipc_open_handle(const void* handle, void** base_out);
int moe_ipc_close_handle(void* base);
/* Asynchronous device-to-device copy (either side may be a peer mapping).   */
int moe_copy_async(void* dst, const void* src, size_t bytes, moe_stream_t stream);

/* Fused dispatch: permute x by the token-major map, writing the row of      */
/* (t, e) straight into rank d = e / experts_per_rank's buffer at row        */
/* map[t,e] + expert_deltas[e]. peer_bases: this process's address of every  */
/* rank's buffer (host array of `ranks` entries, ranks <= 8); expert_deltas: */
/* device array of E row shifts (one per expert, so the owner's buffer may   */
/* be source-major or expert-major). Rows outside [0, cap_rows) of the       */
/* target buffer are skipped.                                                */
int moe_ep_dispatch(const void* x, const int64_t* row_id_map_te, const int64_t* peer_bases,
                    const int64_t* expert_deltas, int32_t ranks, int32_t experts_per_rank,
                    int64_t cap_rows, int64_t T, int64_t H, int64_t E, int64_t num_rows,
                    moe_stream_t stream);
/* One chunk of the fused dispatch, for overlapping the exchange with the    */
/* grouped GEMMs (the comm/compute overlap of the deep_ep FusedDispatch the   */
/* reference names, kernel_cases/case22_ref_moe_permute_mask_kernel_true.py: */
/* 3-6): as moe_ep_dispatch, restricted to the (t, e) whose local expert     */
/* index e % experts_per_rank is in [local_lo, local_hi). The kernel is      */
/* persistent over tokens with at most max_ctas 128-thread CTAs (0 = one per */
/* token), small enough to run beside a grouped GEMM on another stream.      */
int moe_ep_dispatch_range(const void* x, const int64_t* row_id_map_te, const int64_t* peer_bases,
                          const int64_t* expert_deltas, int32_t ranks, int32_t experts_per_rank,
                          int64_t cap_rows, int64_t T, int64_t H, int64_t E, int64_t num_rows,
                          int32_t local_lo, int32_t local_hi, int32_t max_ctas,
                          moe_stream_t stream);
/* Pull form of the fused dispatch (the same receive rows, loaded by the     */
/* receiver instead of stored by the source; the deep_ep FusedDispatch the    */
/* reference names, kernel_cases/case22_ref_moe_permute_mask_kernel_true.py: */
/* 3-6). Step 1, on every rank: moe_ep_pull_stage copies x [T,H] into this    */
/* rank's peer-shared staging rows and writes row_tokens[r] = t for each      */
/* routed (t, e) with r = map[t,e] < num_rows. Step 2, after a barrier, on    */
/* every rank: moe_ep_dispatch_pull fills recv[0, num_recv): group g =       */
/* le * ranks + s of group_table (int32 [3][num_groups] on the device: first  */
/* receive row, rows, first permuted row of source s for local expert le;    */
/* groups in that order, first rows ascending) takes its rows from source s's */
/* staged rows, each token read from s's row_tokens. Loads outside           */
/* tokens_cap / rows_cap are skipped. H % 8 == 0, H <= 8192; num_groups <=   */
/* 1024.                                                                      */
int moe_ep_pull_stage(const void* x, const int64_t* row_id_map_te, int64_t T, int64_t H, int64_t E,
                      int64_t num_rows, void* staged_rows, int32_t* row_tokens,
                      moe_stream_t stream);
int moe_ep_dispatch_pull(const int64_t* peer_staged_rows, const int64_t* peer_row_tokens,
                         int32_t ranks, int64_t tokens_cap, int64_t rows_cap,
                         const int32_t* group_table, int32_t num_groups, void* recv,
                         int64_t num_recv, int64_t cap_rows, int64_t H, moe_stream_t stream);
/* Fused combine: out[t] = bf16(sum over e ascending of probs[t,e] * row),   */
/* each row read from rank e / experts_per_rank's buffer at map[t,e] +       */
/* expert_deltas[e] (device array); probs null = unweighted. Same arithmetic */
/* as moe_unpermute_mask_token_major. E <= 1024.                             */
int moe_ep_combine(const int64_t* peer_bases, const int64_t* expert_deltas, int32_t ranks,
                   int32_t experts_per_rank, int64_t cap_rows, const int64_t* row_id_map_te,
                   const float* probs, void* out, int64_t T, int64_t H, int64_t E,
                   int64_t num_rows, moe_stream_t stream);

/* f3  Backward of the fused combine for this rank's tokens: for each routed */
/* (t, e), owner d = e / experts_per_rank, row rr = map[t,e] + deltas[e]:     */
/* grad_probs[t,e] = <grad_out[t], rows_d[rr]> in fp32 (rows_d: rank d's fc2  */
/* output, peer_rows[d]) and grad_rows_d[rr] = bf16(probs[t,e] * grad_out[t]) */
/* (peer_grad_rows[d]); grad_probs [T,E] is 0 where unrouted. The same bits  */
/* as moe_combine_backward on the single-GPU layout. The expert-parallel     */
/* form of the deep_ep FusedCombine backward the reference names             */
/* (kernel_cases/case24_ref_moe_unpermute_mask_kernel_false.py:3-6). E <=    */
/* 1024.                                                                      */
int moe_ep_combine_backward(const void* grad_out, const int64_t* row_id_map_te, const float* probs,
                            const int64_t* peer_rows, const int64_t* peer_grad_rows,
                            const int64_t* expert_deltas, int32_t ranks, int32_t experts_per_rank,
                            int64_t cap_rows, float* grad_probs, int64_t T, int64_t H, int64_t E,
                            int64_t num_rows, moe_stream_t stream);

/* Deduplicated dispatch (the token-once-per-rank scheme of the deep_ep       */
/* FusedDispatch the reference names, kernel_cases/case22_ref_moe_permute_    */
/* mask_kernel_true.py:3-6): a token row crosses NVLink once per destination  */
/* rank. Rows for this rank's own experts go straight to                      */
/* peer_bases[my_rank] at map[t,e] + expert_deltas[e]; for every other rank d  */
/* the row is stored once into d's staging rows (peer_stage[d], block of T     */
/* rows per source, slot from an atomic on peer_count[d][my_rank]) with a      */
/* destination-row table (peer_meta[d], int32 [ranks*T, experts_per_rank],     */
/* -1 = not routed). E <= 1024, H <= 8192.                                    */
int moe_ep_dispatch_dedup(const void* x, const int64_t* row_id_map_te, const int64_t* peer_bases,
                          const int64_t* expert_deltas, const int64_t* peer_stage,
                          const int64_t* peer_meta, const int64_t* peer_count, int32_t ranks,
                          int32_t my_rank, int32_t experts_per_rank, int64_t cap_rows, int64_t T,
                          int64_t H, int64_t E, int64_t num_rows, moe_stream_t stream);
/* After every rank's dedup dispatch (a barrier): copies each staged row of   */
/* every other source to the receive rows its table lists (rows outside       */
/* [0, cap_rows) skipped), then zeroes the counters for the next dispatch.    */
int moe_ep_expand(const void* stage, const int32_t* meta, int32_t* count, void* recv,
                  int32_t ranks, int32_t my_rank, int32_t experts_per_rank, int64_t rows_per_src,
                  int64_t cap_rows, int64_t H, moe_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H */
