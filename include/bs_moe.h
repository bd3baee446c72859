/*
 * bs_moe.h — C ABI of the B200 (sm_100a) gpt-oss mixture-of-experts layer.
 *
 * The reference (hareramray/BlockStreamer) is pure Python: its MoE layer is
 * transformers' GptOssMLP with block_streamer.gptoss.MXFP4Experts swapped in.
 * Each entry point below replaces one step of that Python path; the comment on
 * each names the reference lines it replaces.  The Python package
 * blockstreamer_b200 binds these with ctypes and keeps the reference's module
 * API (parameter names, shapes, dtypes) on top.
 *
 * Conventions
 *  - Every pointer is a DEVICE pointer unless stated otherwise; sizes are int64.
 *  - `stream` is a cudaStream_t passed as void*; NULL means the legacy stream.
 *    Every call is asynchronous on `stream` unless stated otherwise.
 *  - Return value: BS_OK (0) or a BS_ERR_* code; bs_last_error_string() gives
 *    the message of the last failure on the calling host thread.
 *  - Tensors are dense, row-major, without padding.  Rows handled by 128-bit or
 *    TMA loads must start on 16-byte boundaries (checked: BS_ERR_MISALIGNED).
 *  - Packed expert weights use the checkpoint layout:
 *      blocks [E, rows, G, 16] uint8  (two e2m1 codes per byte, low nibble first)
 *      scales [E, rows, G]     uint8  (e8m0, value 2^(s-127))
 *    with G = K / 32 groups along the contraction dimension K.
 *  - Permuted ("dispatched") rows are grouped by expert: expert e owns rows
 *    [expert_offsets[e], expert_offsets[e+1]) of x_perm / h / y.
 */
#ifndef BS_MOE_H
#define BS_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum bs_status {
  BS_OK = 0,
  BS_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad shape or dtype code            */
  BS_ERR_MISALIGNED = 2,       /* a pointer or row pitch is not 16-byte aligned     */
  BS_ERR_CAPACITY = 3,         /* workspace too small / size beyond a fixed maximum */
  BS_ERR_CUDA = 4,             /* a CUDA runtime call failed                        */
  BS_ERR_TIMEOUT = 5,          /* a bounded device-side wait ran out (see status)   */
  BS_ERR_UNSUPPORTED = 6       /* device is not sm_100 / feature not built          */
};

enum bs_dtype { BS_BF16 = 0, BS_F32 = 1, BS_I32 = 2, BS_I64 = 3 };

enum bs_algo {
  BS_ALGO_AUTO = 0,     /* pick by tokens per expert                                  */
  BS_ALGO_GEMV = 1,     /* CUDA-core dequant-GEMV (decode shapes, HBM-bound)          */
  BS_ALGO_TCGEN05 = 2,  /* tcgen05/TMEM grouped GEMM (prefill shapes)                 */
  BS_ALGO_MX = 3,       /* bs_moe_forward only, T <= 64: tcgen05 block-scaled MMAs on  */
                        /* the e2m1 codes (activations as four e2m1 terms)            */
  BS_ALGO_FUSED = 4,    /* bs_moe_forward only, T <= 8, on request: the whole layer in */
                        /* ONE cooperative persistent kernel                           */
  BS_ALGO_TCGEN05_PAIR = 5  /* on request: the grouped GEMM run by CTA pairs          */
                            /* (tcgen05.mma.cta_group::2, M = 256 weight rows); same   */
                            /* results as BS_ALGO_TCGEN05, measured slower at gpt-oss  */
                            /* shapes                                                  */
};

/* Library identity. */
int bs_version(void);
const char* bs_last_error_string(void);

/* Reads (and with clear != 0, resets) the device status word of the current
 * device: 0 when no kernel reported a problem, else the first BS_ERR_* a kernel
 * recorded (e.g. BS_ERR_TIMEOUT from a bounded mbarrier wait).  Synchronizes
 * `stream`.  Host-side out pointer. */
int bs_device_status(int* out_status, int clear, void* stream);

/* MXFP4 -> bf16 dequantization.
 * Replaces block_streamer/gptoss.py:24-42 (dequantize_expert), which calls
 * transformers integrations/mxfp4.py:333-355 (convert_moe_packed_tensors).
 * out: [E, G*32, rows] bf16 when transpose != 0 (the reference's orientation),
 *      [E, rows, G*32] otherwise.  Bit-exact with the reference for every byte
 *      and scale value (exact product, +-inf beyond the bf16 range). */
int bs_dequant_mxfp4(const void* blocks, const void* scales, int64_t experts, int64_t rows,
                     int64_t groups, int transpose, void* out, void* stream);

/* Router: logits = x W^T + b, top-k (descending), softmax over the k values.
 * Replaces transformers models/gpt_oss/modeling_gpt_oss.py:126-130
 * (GptOssTopKRouter.forward).  x [T,H] bf16 or f32 (x_dtype); weight [E,H] and
 * bias [E] f32 or bf16 (w_dtype; bf16 logits are rounded to bf16 before top-k,
 * as the reference computes them in the weight dtype).  Accumulation is fp32:
 * with a workspace, bf16 x and T > 64 the logits come from the tensor cores
 * with the fp32 weight split exactly into three bf16 terms; otherwise from fp32
 * CUDA-core FMAs.  Top-k ties go to the lower expert index.
 * logits [T,E] f32 (may be NULL); scores [T,k] f32; indices [T,k] int32/int64.
 * workspace: bs_router_workspace_bytes(T, H, E, w_dtype) bytes (may be NULL:
 * then the CUDA-core form runs). */
size_t bs_router_workspace_bytes(int64_t T, int64_t H, int64_t E, int w_dtype);
int bs_router(const void* x, int x_dtype, const void* weight, const void* bias, int w_dtype,
              int64_t T, int64_t H, int64_t E, int64_t k, float* logits, float* scores,
              void* indices, int index_dtype, void* workspace, size_t workspace_bytes,
              void* stream);

/* Workspace bytes bs_dispatch needs for (T, k, E). */
size_t bs_dispatch_workspace_bytes(int64_t T, int64_t k, int64_t E);

/* Token permutation (dispatch).  Replaces block_streamer/gptoss.py:143-154
 * (one_hot / nonzero / where / gather), without any host synchronization.
 * indices [T,k] int32 or int64 (index_dtype) in [0, E).
 * Outputs: expert_offsets [E+1] int32 (exclusive scan of per-expert row counts;
 * offsets[E] = T*k), row_of_slot [T*k] int32 (permuted row of slot (t, s)),
 * token_of_row [T*k] int32, and, when x != NULL, x_perm [T*k, H] bf16 with
 * x_perm[row_of_slot[t*k+s]] = x[t].  Within an expert, rows follow (token, slot)
 * order, so the permutation is deterministic. */
int bs_dispatch(const void* indices, int index_dtype, int64_t T, int64_t k, int64_t E,
                const void* x, int64_t H, int32_t* expert_offsets, int32_t* row_of_slot,
                int32_t* token_of_row, void* x_perm, void* workspace, size_t workspace_bytes,
                void* stream);

/* Allocation-free dispatch: the same outputs as bs_dispatch, with its scratch
 * held in a fixed 512 KiB device array inside the library instead of a caller
 * workspace.  No counterpart in the reference (its dispatch is Python that
 * allocates freely).  It serves callers that cannot allocate device memory
 * where they dispatch: serving loops that must not stall on the device-wide
 * synchronization cudaMalloc/cudaFree imply, runtimes whose pools own all
 * device memory, and ctypes/cgo/JNI callers without a device allocator to
 * hand a workspace from.
 * Limits: 2 * ceil(T/256) * E * 4 bytes <= 512 KiB (e.g. T <= 65536 tokens
 * with E <= 256), else BS_ERR_CAPACITY.  It calls no allocating routine.  The
 * first call on each device looks up the array's device address with that
 * device current and caches it for the process (make that first call before
 * any stream capture; after a cudaDeviceReset the cached address is stale, so
 * do not use this entry point in a process that resets a device it used).
 * Every call on a device shares the one array: calls whose kernels overlap on
 * the GPU (different streams without ordering) race and give wrong results;
 * the array keeps the last call's contents, which every call fully rewrites
 * before reading. */
int bs_dispatch_noalloc(const void* indices, int index_dtype, int64_t T, int64_t k, int64_t E,
                        const void* x, int64_t H, int32_t* expert_offsets, int32_t* row_of_slot,
                        int32_t* token_of_row, void* x_perm, void* stream);

/* Grouped gate_up projection + bias + clamped, interleaved SwiGLU.
 * Replaces block_streamer/gptoss.py:158-166 with _apply_gate (130-135):
 *   g = x_perm[rows of e] @ dequant(W_gu[e]) + b_gu[e]        (fp32 accumulate)
 *   gate = min(g[:, 0::2], limit); up = clamp(g[:, 1::2], -limit, limit)
 *   h = (up + 1) * gate * sigmoid(alpha * gate)               -> bf16 [rows, I]
 * x_perm [rows_total, H] bf16; blocks [E, 2I, H/32, 16]; scales [E, 2I, H/32];
 * bias [E, 2I] (bias_dtype bf16 or f32); h [rows_total, I] bf16.
 * max_rows_per_expert bounds the tile schedule (use rows_total when unknown). */
int bs_moe_gate_up(const void* x_perm, const int32_t* expert_offsets, int64_t rows_total,
                   int64_t max_rows_per_expert, int64_t E, int64_t H, int64_t I,
                   const void* blocks, const void* scales, const void* bias, int bias_dtype,
                   float alpha, float limit, void* h, int algo, void* stream);

/* Grouped down projection + bias.  Replaces block_streamer/gptoss.py:167-174:
 *   y = h[rows of e] @ dequant(W_d[e]) + b_d[e]   -> bf16 [rows_total, H]
 * blocks [E, H, I/32, 16]; scales [E, H, I/32]; bias [E, H]. */
int bs_moe_down(const void* h, const int32_t* expert_offsets, int64_t rows_total,
                int64_t max_rows_per_expert, int64_t E, int64_t H, int64_t I, const void* blocks,
                const void* scales, const void* bias, int bias_dtype, void* y, int algo,
                void* stream);

/* Weighted combine and un-permute.  Replaces block_streamer/gptoss.py:175-176:
 *   out[t] = bf16( sum_s weights[t,s] * y[row_of_slot[t*k+s]] )   (fp32 sum)
 * y [T*k, H] bf16; weights [T,k] f32; out [T,H] bf16. */
int bs_combine(const void* y, const int32_t* row_of_slot, const float* weights, int64_t T,
               int64_t k, int64_t H, void* out, void* stream);

/* Expert parallelism: regroup the rows an all-to-all delivered.
 * No single-GPU counterpart in the reference (it has no expert parallelism);
 * it serves the multi-GPU form of block_streamer/gptoss.py:149-176.
 * recv_counts [R, El] int32 (device): rows from source rank s for local expert e,
 * laid out source-major in x_recv [rows, H] bf16.  Writes x_grouped [rows, H]
 * in expert-major order (within an expert: by source rank, then arrival order),
 * expert_offsets [El+1] and row_map [rows] (received row -> grouped row).
 * x_recv/x_grouped may both be NULL to compute only the maps. */
int bs_ep_regroup(const int32_t* recv_counts, int64_t R, int64_t El, const void* x_recv,
                  int64_t rows, int64_t H, void* x_grouped, int32_t* expert_offsets,
                  int32_t* row_map, void* stream);

/* dst[i] = src[row_map[i]] for i < rows, rows of H bf16 (undoes bs_ep_regroup). */
int bs_gather_rows(const void* src, const int32_t* row_map, int64_t rows, int64_t H, void* dst,
                   void* stream);

/* Expert-parallel exchange over peer memory (NVLink), the B200 form of the
 * all-to-all steps around block_streamer/gptoss.py:149-176 when the experts are
 * sharded over R GPUs (the reference has no distributed backend): no host
 * synchronization, no library collective, plain peer stores (no multicast).
 * Set-up, once per rank (collective over the ranks by the caller):
 *   bs_ep_p2p_bytes(R, E, H, cap_rows, src_rows) -> bytes of the rank's
 *     exchange buffer; src_rows = max dispatched rows per rank (tokens * k),
 *     cap_rows >= R * src_rows rows this rank's experts may receive;
 *   bs_ep_p2p_alloc(bytes, &base, handle[64]) allocates it (cudaMalloc,
 *     zeroed) and returns its CUDA IPC handle; exchange the handles between
 *     the ranks; bs_ep_p2p_open(peer handle, &peer_base) maps a peer's buffer;
 *   the caller places the R bases (its own at index me) in a device array.
 *   bs_ep_p2p_close / bs_ep_p2p_free undo them (free after every peer closed).
 * bs_ep_p2p_layout gives the byte offsets of recv [cap_rows, H] bf16 (the rows
 * this rank's experts process, expert-major, then by source rank) and yback
 * [src_rows, H] bf16 (this rank's dispatched rows' expert results, in its
 * dispatch order) inside a buffer.
 * Per layer call (each rank counts its calls on the device, so the calls may
 * be captured in a CUDA graph and replayed):
 *   bs_ep_p2p_dispatch: from this rank's dispatch (bs_dispatch with x NULL:
 *     expert_offsets [E+1] over GLOBAL experts, token_of_row) and its tokens
 *     x [T, H] bf16, sends every row to its expert's rank; when it returns on
 *     the stream, recv holds every source's rows and local_offsets [E/R + 1]
 *     their expert offsets;
 *   (run gate_up + down on recv with local_offsets, results [cap_rows, H])
 *   bs_ep_p2p_return: sends each result row back to its source's yback; when
 *     it returns on the stream, this rank's yback is complete (combine it with
 *     row_of_slot).
 * Every wait for a peer is bounded (~2 s); a timeout is reported through
 * bs_device_status as BS_ERR_TIMEOUT.
 * Sizes: every rank must dispatch at most src_rows rows (tokens * k <=
 * src_rows, i.e. expert_offsets[E] <= src_rows).  The kernels enforce it: a
 * rank with more rows sends none (its peers see zero rows from it), and every
 * row that would land beyond the destination's cap_rows, or a result beyond
 * its source's src_rows (each rank publishes its own sizes in its buffer), is
 * skipped; each case records BS_ERR_CAPACITY in the status word, so a wrong
 * size never writes outside a peer's buffer. */
size_t bs_ep_p2p_bytes(int64_t R, int64_t E, int64_t H, int64_t cap_rows, int64_t src_rows);
int bs_ep_p2p_layout(int64_t R, int64_t E, int64_t H, int64_t cap_rows, int64_t src_rows,
                     size_t* recv_offset, size_t* yback_offset);
int bs_ep_p2p_alloc(size_t bytes, void** base, void* ipc_handle);
int bs_ep_p2p_open(const void* ipc_handle, void** peer_base);
int bs_ep_p2p_close(void* peer_base);
int bs_ep_p2p_free(void* base);
int bs_ep_p2p_dispatch(const void* x, int64_t H, const int32_t* expert_offsets,
                       const int32_t* token_of_row, void* my_base, const uint64_t* peer_bases,
                       int64_t R, int64_t E, int64_t me, int64_t cap_rows, int64_t src_rows,
                       int32_t* local_offsets, void* stream);
int bs_ep_p2p_return(const void* y, int64_t H, void* my_base, const uint64_t* peer_bases,
                     int64_t R, int64_t E, int64_t me, int64_t cap_rows, int64_t src_rows,
                     void* stream);

/* One expert projection without activation: out[m, N] = x[m, K] @ dequant(W) (+ bias).
 * Replaces block_streamer/gptoss.py:74-75 (mxfp4_matmul forward) for one expert:
 * blocks [N, K/32, 16], scales [N, K/32], x [m, K] bf16, out [m, N] bf16;
 * bias [N] bf16 or NULL. */
int bs_mxfp4_matmul(const void* x, int64_t m, int64_t K, const void* blocks, const void* scales,
                    int64_t N, const void* bias, void* out, int algo, void* stream);

/* Whole layer: router (when router weights are given) or caller routing,
 * dispatch, gate_up+SwiGLU, down, combine.  Replaces GptOssMLP.forward
 * (modeling_gpt_oss.py:140-146) with MXFP4Experts.forward (gptoss.py:137-177).
 *  - router_weight/router_bias non-NULL: computes scores/indices into the
 *    caller's `scores` [T,k] f32 and `indices` [T,k] int32 buffers.
 *  - router_weight NULL: `scores` and `indices` are inputs.
 *  - algo BS_ALGO_FUSED (T <= 8, only when requested; H, I multiples of 64
 *    up to 4096, k <= 8, alpha > 0, limit <= 180, 16-byte aligned weights):
 *    router, top-k, dispatch, gate_up + SwiGLU, down and combine in one
 *    cooperative launch with one CTA per SM, every SM streaming its slice of
 *    the routed experts' packed weights (a 1-D bulk copy per expert run) into
 *    shared memory; grid-wide steps between the phases are bounded waits.
 *  - algo BS_ALGO_MX (T <= 64; what BS_ALGO_AUTO picks there): the
 *    decode path -- four launches chained with programmatic dependent launch;
 *    the expert projections run on tcgen05 block-scaled MMAs that read the
 *    e2m1 codes and e8m0 scales as stored.
 * Workspace: bs_moe_workspace_bytes(T, H, I, E, k) (covers every algo). */
size_t bs_moe_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k);
int bs_moe_forward(const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k,
                   const void* router_weight, const void* router_bias, int router_dtype,
                   float* scores, int32_t* indices,
                   const void* gate_up_blocks, const void* gate_up_scales, const void* gate_up_bias,
                   const void* down_blocks, const void* down_scales, const void* down_bias,
                   int bias_dtype, float alpha, float limit, void* out, void* workspace,
                   size_t workspace_bytes, int algo, void* stream);

/* Decode-shape layer: bs_moe_forward with BS_ALGO_MX (T <= 64 tokens; H and I
 * multiples of 64; blocks and scales 16-byte aligned): router, top-k and
 * dispatch, gate_up + SwiGLU and down on tcgen05 block-scaled MMAs over the
 * stored e2m1 codes, combine -- four launches chained with programmatic
 * dependent launch.  Replaces the same reference lines as bs_moe_forward
 * (modeling_gpt_oss.py:140-146 with gptoss.py:137-177) at decode sizes.
 * Workspace: bs_moe_workspace_bytes. */
int bs_moe_decode(const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k,
                  const void* router_weight, const void* router_bias, int router_dtype,
                  float* scores, int32_t* indices,
                  const void* gate_up_blocks, const void* gate_up_scales, const void* gate_up_bias,
                  const void* down_blocks, const void* down_scales, const void* down_bias,
                  int bias_dtype, float alpha, float limit, void* out, void* workspace,
                  size_t workspace_bytes, void* stream);

/* Backward of the expert layer: dL/dx and dL/d routing weights of
 *   out[t] = sum_s weights[t,s] * (SwiGLU(x[t] @ W_gu[e]^T + b_gu[e]) @ W_d[e]^T + b_d[e]),
 *   e = indices[t,s]  -- i.e. autograd through block_streamer/gptoss.py:137-177
 * with _MXFP4Matmul.backward (gptoss.py:64-71), which the reference runs as a
 * per-expert loop over densely dequantized weights with host syncs.  Here:
 * dispatch, the gate_up pre-activation, h and y recomputed by the forward
 * kernels, dL/dw and dy in one pass, then two TRANSPOSED tcgen05 grouped
 * GEMMs over the packed weights (dg = SwiGLU'(g) * (dy @ W_d), dx_perm =
 * dg @ W_gu) and an fp32 sum over each token's slots; no host sync.
 * x [T,H] bf16; indices [T,k] int32; weights [T,k] f32; grad_out [T,H] bf16
 * or f32 (grad_dtype); grad_x [T,H] f32 and grad_weights [T,k] f32 are
 * written (not accumulated).  H and 2I multiples of 64.
 * Workspace: bs_moe_backward_workspace_bytes(T, H, I, E, k). */
size_t bs_moe_backward_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k);
int bs_moe_backward(const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k,
                    const int32_t* indices, const float* weights, const void* grad_out, int grad_dtype,
                    const void* gate_up_blocks, const void* gate_up_scales, const void* gate_up_bias,
                    const void* down_blocks, const void* down_scales, const void* down_bias,
                    int bias_dtype, float alpha, float limit, float* grad_x, float* grad_weights,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Backward of the router (transformers modeling_gpt_oss.py:126-130: logits =
 * x W^T + b in the weight dtype, top-k, softmax over the k): from
 * grad_scores [T,k] f32 and the forward's scores/indices, ACCUMULATES
 * dL/dx into grad_x [T,H] f32 and, when non-NULL, dL/dW into grad_weight
 * [E,H] f32 and dL/db into grad_bias [E] f32 (atomics).  x bf16 or f32
 * (x_dtype), weight bf16 or f32 (w_dtype). */
int bs_router_backward(const void* x, int x_dtype, int64_t T, int64_t H, int64_t E, int64_t k,
                       const void* weight, int w_dtype, const float* scores, const int32_t* indices,
                       const float* grad_scores, float* grad_x, float* grad_weight, float* grad_bias,
                       void* stream);

/* dL/dx of one expert projection (bs_mxfp4_matmul): grad_x [m,K] bf16 =
 * grad_out [m,N] bf16 @ dequant(W) with W = blocks [N,K/32,16], scales
 * [N,K/32] -- block_streamer/gptoss.py:64-71 without the dense weight (the
 * transposed tcgen05 GEMM over the packed codes).  N a multiple of 64.
 * Workspace: bs_mxfp4_matmul_backward_workspace_bytes(N, K). */
size_t bs_mxfp4_matmul_backward_workspace_bytes(int64_t N, int64_t K);
int bs_mxfp4_matmul_backward(const void* grad_out, int64_t m, int64_t N, const void* blocks,
                             const void* scales, int64_t K, void* grad_x, void* workspace,
                             size_t workspace_bytes, void* stream);

/* RMSNorm of the gpt-oss decoder layer.  Replaces transformers
 * models/gpt_oss/modeling_gpt_oss.py GptOssRMSNorm.forward:
 *   out = bf16(weight * (float(x) * rsqrt(mean(float(x)^2) + eps)))
 * x, out [T, H] bf16 (H a multiple of 8, 16-byte aligned); weight [H] bf16 or
 * f32 (w_dtype). */
int bs_rmsnorm(const void* x, int64_t T, int64_t H, const void* weight, int w_dtype, float eps,
               void* out, void* stream);

/* The MoE half of a gpt-oss decoder layer, fused around the layer: replaces
 * GptOssDecoderLayer.forward's "Fully Connected" part (modeling_gpt_oss.py):
 *   out = x + mlp(post_attention_layernorm(x))
 * = bs_rmsnorm into the workspace, then bs_moe_forward on the normalized rows,
 * whose final combine also adds the residual x (bf16 + bf16, as the reference
 * adds two bf16 tensors).  Same arguments as bs_moe_forward plus the norm
 * weight [H] (norm_dtype bf16 or f32) and eps; out must not alias x.
 * Workspace: bs_moe_block_workspace_bytes(T, H, I, E, k). */
size_t bs_moe_block_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k);
int bs_moe_block_forward(const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k,
                         const void* norm_weight, int norm_dtype, float eps,
                         const void* router_weight, const void* router_bias, int router_dtype,
                         float* scores, int32_t* indices,
                         const void* gate_up_blocks, const void* gate_up_scales, const void* gate_up_bias,
                         const void* down_blocks, const void* down_scales, const void* down_bias,
                         int bias_dtype, float alpha, float limit, void* out, void* workspace,
                         size_t workspace_bytes, int algo, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BS_MOE_H */
