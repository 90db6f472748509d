/*
 * moe_b200.h - C ABI of the B200 (sm_100a) mixture-of-experts MLP hot path.
 *
 * Every entry point replaces one function of the reference Python/Triton
 * package triton_moe (file:line given beside each declaration).  The ABI uses
 * only plain pointers, sizes and a CUDA stream:
 *   - all tensor pointers are DEVICE pointers, row-major, with the given row
 *     stride in elements;
 *   - integer metadata is int32 on the device;
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); every call is
 *     asynchronous on it and never synchronises the host;
 *   - `status` (nullable) is a device int that kernels set to a negative
 *     MOE_ERR_* code when they detect an error on the device (bad expert id,
 *     capacity overflow, a bounded wait that gave up);
 *   - return value: MOE_OK, or a negative MOE_ERR_* code for a host-side
 *     argument or launch error.
 * dtype codes: MOE_DTYPE_BF16 / MOE_DTYPE_F16 / MOE_DTYPE_F32 everywhere; the
 * GEMMs run bf16/fp16 operands on the kind::f16 tensor-core MMA and fp32
 * operands on the kind::tf32 MMA (the reference's default precision for fp32
 * dots), always with fp32 accumulation.
 */
#ifndef MOE_B200_H_
#define MOE_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define MOE_API __attribute__((visibility("default")))
#else
#define MOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_OK 0
#define MOE_ERR_BAD_ARG (-1)
#define MOE_ERR_UNSUPPORTED (-2)
#define MOE_ERR_CUDA (-3)
#define MOE_ERR_TIMEOUT (-4)
#define MOE_ERR_CAPACITY (-5)
#define MOE_ERR_BAD_EXPERT (-6)
#define MOE_ERR_COMM (-7) /* NCCL missing or an NCCL call failed */

#define MOE_DTYPE_BF16 0
#define MOE_DTYPE_F16 1
#define MOE_DTYPE_F32 2

#define MOE_TILE_PAIR 0x200 /* tile_n flag: 256-row tiles on SM pairs */
/* tile_n field: run the launch on at most n persistent CTAs (0 = one per SM),
 * e.g. to leave SMs to communication kernels running alongside */
#define MOE_TILE_CTAS(n) ((n) << 16)
/* Grouped-GEMM tile order: a launch with at least 8 tiles per CTA takes its
 * tiles by ticket from a counter the library keeps per (device, stream) --
 * allocated at the first such call on that stream outside graph capture and
 * zero again after every launch -- so launches ordered on one stream share it
 * and launches on different streams never do.  A graph captured on a stream
 * uses that stream's counter: replay it where it cannot overlap other
 * launches of that stream.  Fewer tiles, CTA pairs, or capture on a stream
 * without a counter: round-robin tiles. */

#define MOE_ACT_NONE 0
#define MOE_ACT_RELU_SQUARED 1
#define MOE_ACT_SWIGLU 2 /* moe_grouped_gemm_up_swiglu */

#define MOE_ROUND_UP 0
#define MOE_ROUND_DOWN 1
#define MOE_ROUND_NEAREST 2

/* Library identification and error text. */
MOE_API const char* moe_version(void);
MOE_API const char* moe_status_string(int status);

/* Time limit, in nanoseconds, of every device-side wait of the grouped-GEMM
 * kernels launched after this call (an mbarrier wait, or a fused up+down
 * launch's wait for its row block of the intermediate); 0 restores the
 * default of 2 s.  A wait that runs out sets MOE_ERR_TIMEOUT in the launch's
 * `status` word, the kernel lets its own copies and MMAs in flight finish,
 * releases its tensor memory and returns; its outputs are then undefined.
 * No counterpart in the reference (its Triton kernels have no device waits);
 * it exists so that a test can make a wait run out quickly.  Process-wide;
 * returns the previous limit. */
MOE_API uint64_t moe_set_wait_timeout_ns(uint64_t ns);

/* Bytes of device workspace moe_route needs for `num_assignments` top-k
 * assignments over `num_experts` experts. */
MOE_API int64_t moe_route_workspace_bytes(int64_t num_assignments, int num_experts);

/*
 * Routing.  Replaces fused_route (triton_moe/kernels/fused_cumsum.py:84-171):
 * stable sort of the flattened top-k expert ids, per-expert histogram,
 * rounded inclusive cumsums (_cumsum_kernel, fused_cumsum.py:20-81) and the
 * drop compaction of the "down"/"nearest" modes (fused_cumsum.py:154-169).
 * Also produces the module's offsets (triton_moe/moe.py:192-202) and the
 * padded-row maps used by the gather/scatter/GEMM kernels.
 *   selected_experts   [num_assignments] int32 (selected_is_int64 = 0) or int64
 *   bin_ids, indices   [num_assignments] (first bins[E-1] entries valid)
 *   tokens_per_expert, bins, padded_bins, padded_tokens_per_expert  [E]
 *   expert_token_offsets [E+1] = [0, padded_bins...]
 *   row_to_assignment  [padded_capacity] or NULL: padded row -> assignment
 *                      index (token*top_k + slot), -1 for padding rows
 *   assignment_to_row  [num_assignments] or NULL: inverse map, -1 if dropped
 *   workspace          moe_route_workspace_bytes(...) bytes of device memory
 */
MOE_API int moe_route(const void* selected_experts, int selected_is_int64, int64_t num_assignments,
              int num_experts, int block_size, int rounding, int32_t* bin_ids, int32_t* indices,
              int32_t* tokens_per_expert, int32_t* bins, int32_t* padded_bins,
              int32_t* expert_token_offsets, int32_t* padded_tokens_per_expert,
              int32_t* row_to_assignment, int64_t padded_capacity, int32_t* assignment_to_row,
              void* workspace, int64_t workspace_bytes, int* status, void* stream);

/*
 * moe_route without a workspace argument.  This entry point has no
 * counterpart in the reference: it exists for callers that cannot allocate
 * device memory themselves -- a plain C or FFI caller that only holds the
 * buffers it was handed, a runtime whose pool or caching allocator already
 * owns the GPU's memory (so an extra cudaMalloc can fail or fragment it), or
 * a latency-critical loop where cudaMalloc/cudaFree would synchronise the
 * device.  It allocates nothing: the histogram scratch is a fixed 256 KiB
 * array of device memory inside the library (room for the largest scratch
 * moe_route can need: 256 units x 256 experts x 4 bytes), held by every GPU
 * that loads the library until the process exits.  Limits are those of
 * moe_route (num_experts <= 256); a problem whose scratch would exceed the
 * array is rejected with MOE_ERR_CAPACITY.  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress, with that device current);
 * make that first call before any stream capture.  All calls on a device share
 * the array and it keeps the last call's contents (nothing in it needs to
 * start at zero), so calls whose kernels overlap on the same GPU -- e.g. on
 * two streams -- race on it and must be serialised by the caller.  Outputs and
 * their meaning are exactly those of moe_route.
 */
MOE_API int moe_route_no_alloc(const void* selected_experts, int selected_is_int64,
                               int64_t num_assignments, int num_experts, int block_size,
                               int rounding, int32_t* bin_ids, int32_t* indices,
                               int32_t* tokens_per_expert, int32_t* bins, int32_t* padded_bins,
                               int32_t* expert_token_offsets, int32_t* padded_tokens_per_expert,
                               int32_t* row_to_assignment, int64_t padded_capacity,
                               int32_t* assignment_to_row, int* status, void* stream);

/*
 * Top-k expert choice for the router output (triton_moe/moe.py:168-182):
 * router_probs [num_tokens, num_experts] fp32 (sigmoid of the router logits)
 * -> selected_experts [num_tokens, top_k] int32 in descending probability order
 * (torch.topk; equal probabilities go to the lower expert index) and weights
 * [num_tokens, top_k] = p / (sum_k p + 1e-20) when normalize, else p, rounded
 * to weights_dtype.  num_experts <= 256, top_k <= 32.
 */
MOE_API int moe_router_topk(const float* router_probs, int64_t num_tokens, int num_experts,
                            int top_k, int normalize, void* weights, int weights_dtype,
                            int32_t* selected_experts, void* stream);

/*
 * Fused router head (triton_moe/moe.py:165-182 and the per-token part of the
 * auxiliary losses, moe.py:253-268).  From router_logits [num_tokens,
 * num_experts] (logits_dtype) in one pass:
 *   router_probs [T, E] fp32 = sigmoid(logits);
 *   selected_experts / weights as moe_router_topk;
 *   lse [T] fp32 = logsumexp(logits_t) with torch's rounding chain in the
 *   logits dtype; workspace (moe_router_head_workspace_floats floats):
 *   per-block partial sums for the losses.
 * The workspace also receives each expert's selection count.
 * moe_aux_losses then forms losses[0] = router_z_loss (mean lse^2, rounded to
 * the logits dtype), losses[1] = load_balance_loss = sum_e lb_coef[e] * f_i[e]
 * * p_i[e], losses[2] = compute_loss = mean_t sum_e probs * widths_normalized,
 * f_i [E] = tokens_per_expert / sum (f_dtype) and p_i [E] fp32 = mean probs;
 * z_loss (nullable) receives router_z_loss in the logits dtype.
 * tokens_per_expert may be NULL: the head's own selection counts are used
 * (equal to fused_route's tokens_per_expert for the same selections), so the
 * losses do not wait for routing.
 */
MOE_API int64_t moe_router_head_workspace_floats(int64_t num_tokens, int num_experts);
MOE_API int moe_router_head(const void* router_logits, int logits_dtype, int64_t num_tokens,
                            int num_experts, int top_k, int normalize,
                            const float* widths_normalized, float* router_probs, void* weights,
                            int weights_dtype, int32_t* selected_experts, float* lse,
                            float* workspace, void* stream);
/*
 * moe_router_head and moe_aux_losses in one launch (no counterpart in the
 * reference, which computes these in torch): the head also counts each
 * expert's selections (= tokens_per_expert), and its last block to finish
 * forms losses / f_i / p_i / z_loss as moe_aux_losses does.  f_i has the
 * weights dtype.  ticket: a device word that is zero before the first call;
 * every call leaves it zero again.  Calls sharing a ticket must not overlap.
 */
MOE_API int moe_router_head_losses(const void* router_logits, int logits_dtype,
                                   int64_t num_tokens, int num_experts, int top_k, int normalize,
                                   const float* widths_normalized, float* router_probs,
                                   void* weights, int weights_dtype, int32_t* selected_experts,
                                   float* lse, float* workspace, const float* lb_coef,
                                   float* losses, void* f_i, float* p_i, void* z_loss,
                                   unsigned* ticket, void* stream);
MOE_API int moe_aux_losses(const float* workspace, int64_t num_tokens, int num_experts,
                           const int32_t* tokens_per_expert, const float* lb_coef,
                           int logits_dtype, float* losses, void* f_i, int f_dtype, float* p_i,
                           void* z_loss, void* stream);

/*
 * Padded-row maps from the reference's sorted-order metadata (indices,
 * bin_ids, bins, padded_bins as returned by fused_route).  The row arithmetic
 * is that of _padded_gather_kernel (triton_moe/kernels/gather.py:29-50).
 * Either output may be NULL.
 */
MOE_API int moe_build_row_map(const int32_t* indices, const int32_t* bin_ids, const int32_t* bins,
                      const int32_t* padded_bins, int64_t num_kept, int64_t padded_rows,
                      int32_t* row_to_assignment, int64_t num_assignments,
                      int32_t* assignment_to_row, int* status, void* stream);

/* precompute_gather_map (triton_moe/kernels/grouped_gemm.py:104-149):
 * gather_map[r] = row_to_assignment[r] / top_k, padding rows 0. */
MOE_API int moe_gather_map(const int32_t* row_to_assignment, int64_t padded_rows, int top_k,
                   int32_t* gather_map, void* stream);

/*
 * Padded gather.  out[r] = x[row_map[r] / map_div] (* weights[row_map[r]] when
 * weights != NULL); rows with a negative map entry are written as zeros.
 * Rows r >= *padded_rows_device (when non-NULL) are left untouched.
 * Replaces padded_gather (triton_moe/kernels/gather.py:63-116, map_div =
 * top_k), _weighted_padded_gather (gather.py:177-218) and the fused-gather
 * row indirection of the GEMMs (grouped_gemm.py:270-273, map_div = 1).
 */
MOE_API int moe_padded_gather(const void* x, int64_t ld_x, int64_t hidden, const int32_t* row_map,
                      int map_div, int64_t padded_rows, const int32_t* padded_rows_device,
                      const void* weights, void* out, int64_t ld_out, int dtype, void* stream);

/*
 * Weighted top-k combine.  out[t] = sum_j round(y[assignment_to_row[t*k+j]] *
 * weights[t*k+j]); weights == NULL means unit weights.  Replaces
 * padded_scatter (triton_moe/kernels/scatter.py:72-135) without the
 * [T, k, H] temporary.
 */
MOE_API int moe_padded_scatter(const void* y, int64_t ld_y, int64_t hidden,
                       const int32_t* assignment_to_row, int64_t num_tokens, int top_k,
                       const void* weights, void* out, int64_t ld_out, int dtype, void* stream);

/* relu^2 derivative: grad_act = pre > 0 ? grad_out * 2 * pre : 0, rounded to
 * dtype (triton_moe/kernels/grouped_gemm.py:751-766). */
MOE_API int moe_relu_squared_grad(const void* grad_out, const void* pre_act, int64_t rows, int64_t cols,
                          int64_t ld, void* grad_act, int dtype, void* stream);

/*
 * Grouped GEMMs.  Common arguments:
 *   expert_token_offsets  [E+1] row offsets of each expert's (padded) rows
 *   expert_weight_offsets [E+1] offsets of each expert's columns of w1 /
 *                         rows of w2
 *   tokens_per_expert     [E] or NULL: caps the rows computed per expert
 *   hidden                hidden size H; w1 is [H, total_width], w2 is
 *                         [total_width, H], both contiguous
 *   rows                  rows of the token-space operands (allocation size)
 *   tile_n                N tile 128 or 256 (0 = choose); OR MOE_TILE_PAIR for
 *                         256-row tiles computed by SM pairs (2-CTA clusters,
 *                         cta_group::2 MMAs) instead of 128-row tiles; OR
 *                         MOE_TILE_CTAS(n) to cap the persistent grid at n CTAs
 * Every expert width and every expert row count used as a reduction length
 * must be a multiple of 16; H must be a multiple of 16.
 */

/* grouped_gemm_up (triton_moe/kernels/grouped_gemm.py:378-477, kernel :212-368):
 * out = act(x @ w1_e); with MOE_ACT_RELU_SQUARED and pre_act != NULL also
 * pre_act = relu(x @ w1_e).  Columns >= w_e of out / pre_act are not written. */
MOE_API int moe_grouped_gemm_up(const void* x, int64_t rows, int64_t ld_x, const void* w1,
                        int64_t hidden, int64_t total_width,
                        const int32_t* expert_token_offsets,
                        const int32_t* expert_weight_offsets, const int32_t* tokens_per_expert,
                        int num_experts, int activation, void* out, void* pre_act,
                        int64_t ld_out, int dtype, int tile_n, int* status, void* stream);

/* grouped_gemm_up with activation "swiglu" (grouped_gemm.py:270-358,
 * ACTIVATION == 2): expert e's w1 columns are its gate block then its up block,
 * so expert_weight_offsets step by 2 w_e and total_width = sum 2 w_e.
 * out[rows_e, :w_e] = silu(x @ gate_e) * (x @ up_e) from the fp32 accumulators;
 * gate (the reference's pre_act) and up (nullable) receive the rounded
 * projections for the backward.  out / gate / up share ld_out. */
MOE_API int moe_grouped_gemm_up_swiglu(const void* x, int64_t rows, int64_t ld_x, const void* w1,
                                       int64_t hidden, int64_t total_width,
                                       const int32_t* expert_token_offsets,
                                       const int32_t* expert_weight_offsets,
                                       const int32_t* tokens_per_expert, int num_experts,
                                       void* out, void* gate, void* up, int64_t ld_out,
                                       int dtype, int tile_n, int* status, void* stream);

/* SwiGLU backward through the activation (the reference's is a placeholder,
 * grouped_gemm.py:768-789): with s = sigmoid(gate),
 * grad_act[r, 0:w_e) = g * up * s * (1 + gate (1 - s)) and
 * grad_act[r, w_e:2 w_e) = g * gate * s for the rows of each expert e
 * (expert_weight_offsets in the 2 w_e layout); moe_grouped_gemm_up_dx / _dw /
 * _backward over that layout then give dX and dW1. */
MOE_API int moe_swiglu_grad(const void* grad_out, const void* gate, const void* up, int64_t rows,
                            int64_t ld, const int32_t* expert_token_offsets,
                            const int32_t* expert_weight_offsets, int num_experts,
                            void* grad_act, int64_t ld_act, int dtype, void* stream);

/* grouped_gemm_up (relu^2, saving pre_act) and grouped_gemm_down in ONE
 * persistent launch: inter = relu(x @ w1_e)^2, out = inter @ w2_e.  A down tile
 * starts as soon as every up tile of its 128-row block has stored its rows (a
 * per-block count in `dep`), so the down tiles fill the SMs the up tiles' tail
 * leaves idle instead of waiting for a second launch.  dep: an int32 device
 * buffer of at least moe_up_down_dep_words(rows, num_experts) words, zero
 * before the first call; each call returns it to zero.  Calls on one GPU must
 * not overlap at all (order them on one stream or with events): a down tile
 * waits for other blocks' up tiles, so the whole grid has to be resident, and
 * two overlapping launches could hold SMs against each other until their
 * bounded waits give up (MOE_ERR_TIMEOUT). */
MOE_API int64_t moe_up_down_dep_words(int64_t rows, int num_experts);
MOE_API int moe_grouped_gemm_up_down(const void* x, int64_t rows, int64_t ld_x, const void* w1,
                                     const void* w2, int64_t hidden, int64_t total_width,
                                     const int32_t* expert_token_offsets,
                                     const int32_t* expert_weight_offsets,
                                     const int32_t* tokens_per_expert, int num_experts,
                                     void* inter, void* pre_act, int64_t ld_inter, void* out,
                                     int64_t ld_out, int32_t* dep, int64_t dep_words, int dtype,
                                     int tile_n_width, int tile_n_hidden, int* status,
                                     void* stream);

/* grouped_gemm_down (grouped_gemm.py:586-651, kernel :480-583):
 * out[rows_e] = inter[rows_e, :w_e] @ w2[w_e rows]. */
MOE_API int moe_grouped_gemm_down(const void* inter, int64_t rows, int64_t ld_inter, const void* w2,
                          int64_t hidden, int64_t total_width,
                          const int32_t* expert_token_offsets,
                          const int32_t* expert_weight_offsets,
                          const int32_t* tokens_per_expert, int num_experts, void* out,
                          int64_t ld_out, int dtype, int tile_n, int* status, void* stream);

/* dX half of grouped_gemm_up_backward (grouped_gemm.py:1165-1290, kernel
 * :654-802) with the activation derivative already applied:
 * grad_x[rows_e] = grad_act[rows_e, :w_e] @ w1_e^T. */
MOE_API int moe_grouped_gemm_up_dx(const void* grad_act, int64_t rows, int64_t ld_grad_act,
                           const void* w1, int64_t hidden, int64_t total_width,
                           const int32_t* expert_token_offsets,
                           const int32_t* expert_weight_offsets,
                           const int32_t* tokens_per_expert, int num_experts, void* grad_x,
                           int64_t ld_grad_x, int dtype, int tile_n, int* status, void* stream);

/* dW half of grouped_gemm_up_backward (kernel grouped_gemm.py:805-967):
 * grad_w1[:, w_e cols] = x[rows_e]^T @ grad_act[rows_e, :w_e], reduced over
 * each expert's full row range (experts with no rows get zeros). */
MOE_API int moe_grouped_gemm_up_dw(const void* x, int64_t rows, int64_t ld_x, const void* grad_act,
                           int64_t ld_grad_act, int64_t hidden, int64_t total_width,
                           const int32_t* expert_token_offsets,
                           const int32_t* expert_weight_offsets, int num_experts,
                           void* grad_w1, int dtype, int tile_n, int* status, void* stream);

/* dIntermediate half of grouped_gemm_down_backward (grouped_gemm.py:1293-1390,
 * kernel :970-1063): grad_inter[rows_e, :w_e] = grad_y[rows_e] @ w2_e^T.
 * When pre_act != NULL the relu^2 derivative is fused into the epilogue and
 * `out` receives grad_act = relu2'(pre_act) * round(grad_inter) instead. */
MOE_API int moe_grouped_gemm_down_dinter(const void* grad_y, int64_t rows, int64_t ld_grad_y,
                                 const void* w2, int64_t hidden, int64_t total_width,
                                 const int32_t* expert_token_offsets,
                                 const int32_t* expert_weight_offsets,
                                 const int32_t* tokens_per_expert, int num_experts,
                                 const void* pre_act, int64_t ld_pre, void* out, int64_t ld_out,
                                 int dtype, int tile_n, int* status, void* stream);

/* dW half of grouped_gemm_down_backward (kernel grouped_gemm.py:1066-1162):
 * grad_w2[w_e rows] = inter[rows_e, :w_e]^T @ grad_y[rows_e]. */
MOE_API int moe_grouped_gemm_down_dw(const void* inter, int64_t rows, int64_t ld_inter,
                             const void* grad_y, int64_t ld_grad_y, int64_t hidden,
                             int64_t total_width, const int32_t* expert_token_offsets,
                             const int32_t* expert_weight_offsets, int num_experts,
                             void* grad_w2, int dtype, int tile_n, int* status, void* stream);

/* The whole of grouped_gemm_down_backward (grouped_gemm.py:1293-1390) in one
 * persistent launch: dIntermediate (or, with pre_act, the fused relu^2
 * derivative) and dW2 share one tile list.  tile_n_width / tile_n_hidden are
 * the N tiles of the two problems. */
MOE_API int moe_grouped_gemm_down_backward(
    const void* grad_y, int64_t rows, int64_t ld_grad_y, const void* inter, int64_t ld_inter,
    const void* w2, int64_t hidden, int64_t total_width, const int32_t* expert_token_offsets,
    const int32_t* expert_weight_offsets, const int32_t* tokens_per_expert, int num_experts,
    const void* pre_act, int64_t ld_pre, void* grad_inter, int64_t ld_grad_inter, void* grad_w2,
    int dtype, int tile_n_width, int tile_n_hidden, int* status, void* stream);

/* The GEMMs of grouped_gemm_up_backward (grouped_gemm.py:1165-1290) in one
 * persistent launch: dX and dW1 from the activation gradient grad_act (the
 * relu^2 derivative already applied). */
MOE_API int moe_grouped_gemm_up_backward(
    const void* grad_act, int64_t rows, int64_t ld_grad_act, const void* x, int64_t ld_x,
    const void* w1, int64_t hidden, int64_t total_width, const int32_t* expert_token_offsets,
    const int32_t* expert_weight_offsets, const int32_t* tokens_per_expert, int num_experts,
    void* grad_x, int64_t ld_grad_x, void* grad_w1, int dtype, int tile_n_width,
    int tile_n_hidden, int* status, void* stream);

/*
 * Expert parallelism (EP): the token exchange between the ranks that share
 * one layer's experts.  The reference runs the layer on one GPU
 * (triton_moe/moe.py:185-249: gather -> grouped GEMMs -> scatter); sharded,
 * each rank routes its own tokens (moe_route with block size 1: its rows in
 * expert-sorted order), and
 *   moe_ep_dispatch  (the gather, fused with the transfer) pushes each row
 *                    straight into the padded expert-contiguous layout of
 *                    the expert's owner (the rows the owner's grouped GEMMs
 *                    read), in the owner's memory;
 *   moe_ep_combine   (the scatter, fused with the transfer) forms each
 *                    token's top-k sum from the owners' output rows, read
 *                    from the owners' memory.
 * Owners' layouts live in buffers made with moe_ep_buffer_create and mapped
 * on every rank with moe_ep_buffer_open (CUDA IPC over NVLink); `peers` is a
 * device array of the world's base pointers of one such buffer (this rank's
 * own entry may be its local pointer).  Ranks order their accesses to each
 * other's buffers with moe_ep_barrier on the streams that access them: after
 * the last read of a buffer and before the next write into it, and after the
 * writes and before the reads.
 *
 * Conventions: `owner` is the rank that owns each global expert (host int32
 * for moe_ep_plan, a device copy for the kernels); a rank's local experts are
 * the ids it owns, ascending.  `counts` (host, int32,
 * [world][chunks][num_experts] row-major) holds how many rows every source
 * rank sends to each expert in each chunk (tokens split into chunks that are
 * exchanged one after another, so that one chunk's GEMMs overlap another's
 * transfers): every rank gathers it with moe_ep_gather_counts.  `comm` is an
 * ncclComm_t of the world's ranks (moe_ep_comm_init, or the caller's own);
 * NCCL is loaded at run time (libnccl.so.2, the copy already in the process
 * if there is one).  Every collective call on a communicator must be made by
 * all its ranks in the same order.
 */

/* ncclGetUniqueId: 128 bytes for moe_ep_comm_init, made on one rank and sent
 * to the others by the caller's own means. */
MOE_API int moe_ep_unique_id(void* id);
/* ncclCommInitRank on the current CUDA device; collective over the ranks. */
MOE_API int moe_ep_comm_init(void** comm, const void* id, int world, int rank);
MOE_API int moe_ep_comm_destroy(void* comm);

/* All-gather of every rank's `n` int32 counts (device buffers; `all` holds
 * world * n, in rank order). */
MOE_API int moe_ep_gather_counts(void* comm, const int32_t* mine, int32_t* all, int64_t n,
                                 void* stream);

/* Stream-ordered barrier of the communicator's ranks (an all-reduce of one
 * int32 device word; its value is not meaningful). */
MOE_API int moe_ep_barrier(void* comm, int32_t* word, void* stream);

/* Device buffers other ranks can map: cudaMalloc + a 64-byte CUDA IPC
 * handle; moe_ep_buffer_open maps a peer's handle (peer access enabled on
 * first use), moe_ep_buffer_close unmaps it. */
MOE_API int moe_ep_buffer_create(int64_t bytes, void** ptr, void* ipc_handle);
MOE_API int moe_ep_buffer_free(void* ptr);
MOE_API int moe_ep_buffer_open(const void* ipc_handle, void** ptr);
MOE_API int moe_ep_buffer_close(void* ptr);

/* Host-side plan of the exchange from the gathered counts (no device work).
 * The owner's layout has one region per local expert; a region holds one
 * block per chunk, each with the sources' rows in rank order, rounded up to
 * block_size rows.
 *   src_off    [chunks][num_experts]: first row of (chunk, expert) in this
 *              rank's expert-sorted rows of that chunk
 *   tok_off    [E_local + 1]: the regions (expert_token_offsets of the whole
 *              layout: the weight-gradient GEMMs reduce over all chunks)
 *   chunk_off  [chunks][E_local + 1]: first row of each chunk's block in each
 *              region, last entry = total rows (expert_token_offsets of one
 *              chunk's GEMMs, with chunk_rows as their tokens_per_expert)
 *   chunk_rows [chunks][E_local]: rows of each chunk's block (padded)
 *   recv_off   [world][chunks][E_local]: first row of the block from each
 *              source rank
 * The row of this rank's expert-sorted row i of chunk c (expert e) in its
 * owner's layout is i - src_off[c][e] + the owner's recv_off[rank][c][e's
 * local index]: the `delta` of moe_ep_dispatch / moe_ep_combine.  Padding
 * rows (past a block's received rows) are not written by the exchange;
 * callers zero them. */
MOE_API int moe_ep_plan(int world, int rank, int chunks, int num_experts, int block_size,
                        const int32_t* owner, const int32_t* counts, int64_t* src_off,
                        int32_t* tok_off, int32_t* chunk_off, int32_t* chunk_rows,
                        int64_t* recv_off);

/* Dispatch one chunk: row i < rows of this rank's expert-sorted rows
 * (row_to_assignment[i] = t * top_k + j, expert bin_ids[i], from moe_route
 * with block size 1 over the chunk's assignments) is token t of x (times
 * weights[row_to_assignment[i]] when weights is not NULL, rounded to the
 * storage type: the weighted gather of the backward) and is stored at row
 * i + delta[e] of peers[owner[e]] (row stride ld_peer).  owner [E] int32,
 * delta [E] int64 and peers [world] are device arrays. */
MOE_API int moe_ep_dispatch(const void* x, int64_t ld_x, int64_t hidden,
                            const int32_t* row_to_assignment, int top_k, const void* weights,
                            const int32_t* bin_ids, int64_t rows, const int32_t* owner,
                            const int64_t* delta, void* const* peers, int64_t ld_peer,
                            int dtype, void* stream);

/* Combine one chunk: out[t] = sum_j round(Y(t, j) * weights[t*top_k + j])
 * (unit weights when NULL), summed in fp32 and rounded once, for t <
 * num_tokens, where assignment a = t*top_k + j is at expert-sorted row
 * r = assignment_to_row[a], its expert is e = bin_ids[r] and Y(t, j) is row
 * r + delta[e] of peers[owner[e]]. */
MOE_API int moe_ep_combine(void* const* peers, int64_t ld_peer, const int32_t* owner,
                           const int64_t* delta, const int32_t* bin_ids,
                           const int32_t* assignment_to_row, int64_t num_tokens, int top_k,
                           const void* weights, int64_t hidden, void* out, int64_t ld_out,
                           int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H_ */
