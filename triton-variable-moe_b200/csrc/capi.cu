// extern "C" entry points of libmoe_b200 (declared in include/moe_b200.h).
// Each one validates its host-side arguments, maps the reference operation
// onto the kernels of route.cu / permute.cu / grouped_gemm.cu and launches on
// the caller's stream.
#include <cuda_runtime.h>

#include <cstdint>

#include "moe_b200.h"
#include "grouped_gemm.cuh"
#include "moe_internal.h"

namespace moe {
long long route_workspace_bytes(long long A, int E);
int route(const void* sel, int sel_is_int64, long long A, int E, int bs, int mode,
          int32_t* bin_ids, int32_t* indices, int32_t* tpe, int32_t* bins, int32_t* padded_bins,
          int32_t* tok_off, int32_t* ptpe, int32_t* row_asg, long long p_cap, int32_t* asg_row,
          void* ws, long long ws_bytes, int* status, cudaStream_t st);
int route_static_scratch(const void* sel, int sel_is_int64, long long A, int E, int bs, int mode,
                         int32_t* bin_ids, int32_t* indices, int32_t* tpe, int32_t* bins,
                         int32_t* padded_bins, int32_t* tok_off, int32_t* ptpe, int32_t* row_asg,
                         long long p_cap, int32_t* asg_row, int* status, cudaStream_t st);
int router_topk(const float* probs, long long T, int E, int k, int norm, void* w, int w_dtype,
                int32_t* sel, cudaStream_t st);
int router_head_blocks(long long T);
int router_head(const void* logits, int l_dtype, long long T, int E, int k, int norm,
                const float* widths_norm, float* probs, void* w, int w_dtype, int32_t* sel,
                float* lse, float* partials, int nblocks, const float* lb_coef, float* losses,
                void* f_i, float* p_i, void* z_out, unsigned* ticket, cudaStream_t st);
int aux_finalize(const float* partials, int nblocks, int E, long long T, const int32_t* tpe,
                 const float* lb_coef, int l_dtype, float* losses, void* f_i, int f_dtype,
                 float* p_i, void* z_out, cudaStream_t st);
int gather_rows(const void* x, long long ldx, int H, const int32_t* map, int div,
                long long rows, const int32_t* rows_dev, const void* w, void* out, long long ldo,
                int dtype, cudaStream_t st);
int swiglu_grad(const void* g, const void* gate, const void* up, long long rows, long long ld,
                const int32_t* tok_off, const int32_t* w_off, int E, void* out, long long ld_out,
                int dtype, cudaStream_t st);
int combine_rows(const void* y, long long ldy, int H, const int32_t* asg_row, long long T_tokens,
                 int k, const void* w, void* out, long long ldo, int dtype, cudaStream_t st);
int relu2_grad(const void* g, const void* pre, long long rows, long long cols, long long ld,
               void* out, int dtype, cudaStream_t st);
int build_row_map(const int32_t* indices, const int32_t* bin_ids, const int32_t* bins,
                  const int32_t* padded_bins, long long n_kept, long long p_rows,
                  int32_t* row_asg, long long n_asg, int32_t* asg_row, int* status,
                  cudaStream_t st);
int gather_map_from_rows(const int32_t* row_asg, long long rows, int k, int32_t* gmap,
                         cudaStream_t st);
}  // namespace moe

namespace {

using moe::GemmOperands;
using moe::GroupedGemmDesc;

cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

bool gemm_dtype_ok(int dtype) {
  return dtype == MOE_DTYPE_BF16 || dtype == MOE_DTYPE_F16 || dtype == MOE_DTYPE_F32;
}

int pick_bn(int tile_n, long long n_hint) {
  const int t = tile_n & 0x1FF;
  if (t == 128 || t == 256) return t;
  return (n_hint > 0 && n_hint % 256 == 0) ? 256 : 128;
}
// 2: 256-row tiles on 2-CTA clusters; 1: 128-row tiles on single CTAs.
int pick_pair(int tile_n) { return (tile_n & MOE_TILE_PAIR) ? 2 : 1; }
// MOE_TILE_CTAS(n): run the launch on at most n CTAs (0: one per SM).
int pick_ctas(int tile_n) { return (tile_n >> 16) & 0x7FFF; }

GroupedGemmDesc base_desc(const int32_t* tok_off, const int32_t* tok_cnt, const int32_t* w_off,
                          int E, long long hidden, int* status) {
  GroupedGemmDesc g{};
  g.tok_off = tok_off;
  g.tok_cnt = tok_cnt;
  g.w_off = w_off;
  g.E = E;
  g.cdim = static_cast<int>(hidden);
  g.status = status;
  return g;
}

bool common_ok(long long rows, long long hidden, long long total_width, const int32_t* tok_off,
               const int32_t* w_off, int E) {
  return rows >= 1 && hidden >= 16 && hidden % 16 == 0 && total_width >= 16 &&
         total_width % 16 == 0 && tok_off && w_off && E >= 1 && E <= moe::kMaxGroups;
}

}  // namespace

extern "C" {

uint64_t moe_set_wait_timeout_ns(uint64_t ns) {
  return static_cast<uint64_t>(moe::set_wait_ns(static_cast<unsigned long long>(ns)));
}

const char* moe_version(void) { return "moe_b200 0.1 (sm_100a tcgen05)"; }

const char* moe_status_string(int s) {
  switch (s) {
    case MOE_OK: return "ok";
    case MOE_ERR_BAD_ARG: return "invalid argument";
    case MOE_ERR_UNSUPPORTED: return "unsupported configuration";
    case MOE_ERR_CUDA: return "CUDA error";
    case MOE_ERR_TIMEOUT: return "device-side wait timed out";
    case MOE_ERR_CAPACITY: return "padded row capacity exceeded";
    case MOE_ERR_BAD_EXPERT: return "expert id out of range";
    case MOE_ERR_COMM: return "NCCL unavailable or an NCCL call failed";
    default: return "unknown status";
  }
}

int64_t moe_route_workspace_bytes(int64_t num_assignments, int num_experts) {
  if (num_assignments < 0 || num_experts <= 0) return 0;
  return moe::route_workspace_bytes(num_assignments, num_experts);
}

int moe_route(const void* selected_experts, int selected_is_int64, int64_t num_assignments,
              int num_experts, int block_size, int rounding, int32_t* bin_ids, int32_t* indices,
              int32_t* tokens_per_expert, int32_t* bins, int32_t* padded_bins,
              int32_t* expert_token_offsets, int32_t* padded_tokens_per_expert,
              int32_t* row_to_assignment, int64_t padded_capacity, int32_t* assignment_to_row,
              void* workspace, int64_t workspace_bytes, int* status, void* stream) {
  return moe::route(selected_experts, selected_is_int64, num_assignments, num_experts,
                    block_size, rounding, bin_ids, indices, tokens_per_expert, bins, padded_bins,
                    expert_token_offsets, padded_tokens_per_expert, row_to_assignment,
                    padded_capacity, assignment_to_row, workspace, workspace_bytes, status,
                    S(stream));
}

// Same routing as moe_route, for callers that cannot allocate device memory:
// the histogram scratch lives in a fixed device array inside the library.
int moe_route_no_alloc(const void* selected_experts, int selected_is_int64,
                       int64_t num_assignments, int num_experts, int block_size, int rounding,
                       int32_t* bin_ids, int32_t* indices, int32_t* tokens_per_expert,
                       int32_t* bins, int32_t* padded_bins, int32_t* expert_token_offsets,
                       int32_t* padded_tokens_per_expert, int32_t* row_to_assignment,
                       int64_t padded_capacity, int32_t* assignment_to_row, int* status,
                       void* stream) {
  return moe::route_static_scratch(selected_experts, selected_is_int64, num_assignments,
                                   num_experts, block_size, rounding, bin_ids, indices,
                                   tokens_per_expert, bins, padded_bins, expert_token_offsets,
                                   padded_tokens_per_expert, row_to_assignment, padded_capacity,
                                   assignment_to_row, status, S(stream));
}

int moe_router_topk(const float* router_probs, int64_t num_tokens, int num_experts, int top_k,
                    int normalize, void* weights, int weights_dtype, int32_t* selected_experts,
                    void* stream) {
  return moe::router_topk(router_probs, num_tokens, num_experts, top_k, normalize, weights,
                          weights_dtype, selected_experts, S(stream));
}

int64_t moe_router_head_workspace_floats(int64_t num_tokens, int num_experts) {
  if (num_tokens < 0 || num_experts <= 0) return 0;
  return static_cast<int64_t>(moe::router_head_blocks(num_tokens)) * (2 * num_experts + 2);
}

int moe_router_head(const void* router_logits, int logits_dtype, int64_t num_tokens,
                    int num_experts, int top_k, int normalize, const float* widths_normalized,
                    float* router_probs, void* weights, int weights_dtype,
                    int32_t* selected_experts, float* lse, float* workspace, void* stream) {
  if (num_tokens == 0) return MOE_OK;
  return moe::router_head(router_logits, logits_dtype, num_tokens, num_experts, top_k, normalize,
                          widths_normalized, router_probs, weights, weights_dtype,
                          selected_experts, lse, workspace, moe::router_head_blocks(num_tokens),
                          nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, S(stream));
}

int moe_router_head_losses(const void* router_logits, int logits_dtype, int64_t num_tokens,
                           int num_experts, int top_k, int normalize,
                           const float* widths_normalized, float* router_probs, void* weights,
                           int weights_dtype, int32_t* selected_experts, float* lse,
                           float* workspace, const float* lb_coef, float* losses, void* f_i,
                           float* p_i, void* z_loss, unsigned* ticket, void* stream) {
  if (num_tokens <= 0 || losses == nullptr) return MOE_ERR_BAD_ARG;
  return moe::router_head(router_logits, logits_dtype, num_tokens, num_experts, top_k, normalize,
                          widths_normalized, router_probs, weights, weights_dtype,
                          selected_experts, lse, workspace, moe::router_head_blocks(num_tokens),
                          lb_coef, losses, f_i, p_i, z_loss, ticket, S(stream));
}

int moe_aux_losses(const float* workspace, int64_t num_tokens, int num_experts,
                   const int32_t* tokens_per_expert, const float* lb_coef, int logits_dtype,
                   float* losses, void* f_i, int f_dtype, float* p_i, void* z_loss,
                   void* stream) {
  return moe::aux_finalize(workspace, moe::router_head_blocks(num_tokens), num_experts,
                           num_tokens, tokens_per_expert, lb_coef, logits_dtype, losses, f_i,
                           f_dtype, p_i, z_loss, S(stream));
}

int moe_build_row_map(const int32_t* indices, const int32_t* bin_ids, const int32_t* bins,
                      const int32_t* padded_bins, int64_t num_kept, int64_t padded_rows,
                      int32_t* row_to_assignment, int64_t num_assignments,
                      int32_t* assignment_to_row, int* status, void* stream) {
  if (num_kept < 0 || padded_rows < 0 || num_assignments < 0) return MOE_ERR_BAD_ARG;
  if (num_kept > 0 && (!indices || !bin_ids || !bins || !padded_bins)) return MOE_ERR_BAD_ARG;
  return moe::build_row_map(indices, bin_ids, bins, padded_bins, num_kept, padded_rows,
                            row_to_assignment, num_assignments, assignment_to_row, status,
                            S(stream));
}

int moe_gather_map(const int32_t* row_to_assignment, int64_t padded_rows, int top_k,
                   int32_t* gather_map, void* stream) {
  if (top_k <= 0 || padded_rows < 0) return MOE_ERR_BAD_ARG;
  return moe::gather_map_from_rows(row_to_assignment, padded_rows, top_k, gather_map, S(stream));
}

int moe_padded_gather(const void* x, int64_t ld_x, int64_t hidden, const int32_t* row_map,
                      int map_div, int64_t padded_rows, const int32_t* padded_rows_device,
                      const void* weights, void* out, int64_t ld_out, int dtype, void* stream) {
  if (map_div <= 0 || hidden < 0 || padded_rows < 0 || ld_x < hidden || ld_out < hidden)
    return MOE_ERR_BAD_ARG;
  if (padded_rows > 0 && (!x || !row_map || !out)) return MOE_ERR_BAD_ARG;
  return moe::gather_rows(x, ld_x, static_cast<int>(hidden), row_map, map_div, padded_rows,
                          padded_rows_device, weights, out, ld_out, dtype, S(stream));
}

int moe_padded_scatter(const void* y, int64_t ld_y, int64_t hidden,
                       const int32_t* assignment_to_row, int64_t num_tokens, int top_k,
                       const void* weights, void* out, int64_t ld_out, int dtype, void* stream) {
  if (top_k <= 0 || hidden < 0 || num_tokens < 0 || ld_y < hidden || ld_out < hidden)
    return MOE_ERR_BAD_ARG;
  if (num_tokens > 0 && (!y || !assignment_to_row || !out)) return MOE_ERR_BAD_ARG;
  return moe::combine_rows(y, ld_y, static_cast<int>(hidden), assignment_to_row, num_tokens,
                           top_k, weights, out, ld_out, dtype, S(stream));
}

int moe_relu_squared_grad(const void* grad_out, const void* pre_act, int64_t rows, int64_t cols,
                          int64_t ld, void* grad_act, int dtype, void* stream) {
  if (rows < 0 || cols < 0 || ld < cols) return MOE_ERR_BAD_ARG;
  return moe::relu2_grad(grad_out, pre_act, rows, cols, ld, grad_act, dtype, S(stream));
}

}  // extern "C"

namespace {

struct Built {
  GemmOperands op;
  GroupedGemmDesc g;
  int epi;
  int err;
};

Built bad(int err) {
  Built b{};
  b.err = err;
  return b;
}

Built build_up(const void* x, int64_t rows, int64_t ld_x, const void* w1, int64_t hidden,
               int64_t total_width, const int32_t* tok_off, const int32_t* w_off,
               const int32_t* tpe, int E, int activation, void* out, void* pre_act,
               int64_t ld_out, int tile_n, int* status) {
  if (!common_ok(rows, hidden, total_width, tok_off, w_off, E) || !x || !w1 || !out ||
      ld_x < hidden || ld_out < 16 || ld_out % 8 != 0)
    return bad(MOE_ERR_BAD_ARG);
  if (activation != MOE_ACT_NONE && activation != MOE_ACT_RELU_SQUARED)
    return bad(MOE_ERR_UNSUPPORTED);
  Built b{};
  b.g = base_desc(tok_off, tpe, w_off, E, hidden, status);
  b.g.m_src = moe::DIM_TOKENS;
  b.g.n_src = moe::DIM_WIDTH;
  b.g.k_src = moe::DIM_CONST;
  b.g.a_m_base = moe::BASE_TOK;
  b.g.b_n_base = moe::BASE_WOFF;
  b.g.d_m_base = moe::BASE_TOK;
  b.g.d = out;
  b.g.ldd = ld_out;
  b.g.d_rows = rows;
  b.epi = moe::EPI_STORE;
  if (activation == MOE_ACT_RELU_SQUARED) {
    b.epi = moe::EPI_RELU2;
    b.g.aux = pre_act;  // may be null: only relu(acc)^2 is stored
    b.g.ld_aux = ld_out;
    b.g.aux_rows = rows;
  }
  b.op = GemmOperands{x, rows, hidden, ld_x, 0, w1, hidden, total_width, total_width, 1,
                      pick_bn(tile_n, 0), 0};
  b.op.pair = pick_pair(tile_n);
  b.op.grid = pick_ctas(tile_n);
  return b;
}

// SwiGLU up projection: expert e's w1 columns are its gate block then its up
// block (w_off spacing 2 w_e); out = silu(x @ gate) * (x @ up), gate / up
// optionally stored (rounded) for the backward.
Built build_up_swiglu(const void* x, int64_t rows, int64_t ld_x, const void* w1, int64_t hidden,
                      int64_t total_width, const int32_t* tok_off, const int32_t* w_off,
                      const int32_t* tpe, int E, void* out, void* gate, void* up, int64_t ld_out,
                      int tile_n, int* status) {
  if (!common_ok(rows, hidden, total_width, tok_off, w_off, E) || !x || !w1 || !out ||
      ld_x < hidden || ld_out < 16 || ld_out % 8 != 0)
    return bad(MOE_ERR_BAD_ARG);
  Built b{};
  b.g = base_desc(tok_off, tpe, w_off, E, hidden, status);
  b.g.m_src = moe::DIM_TOKENS;
  b.g.n_src = moe::DIM_HALF_WIDTH;
  b.g.k_src = moe::DIM_CONST;
  b.g.a_m_base = moe::BASE_TOK;
  b.g.b_n_base = moe::BASE_WOFF;
  b.g.d_m_base = moe::BASE_TOK;
  b.g.d = out;
  b.g.ldd = ld_out;
  b.g.d_rows = rows;
  b.g.aux = gate;
  b.g.ld_aux = ld_out;
  b.g.aux_rows = rows;
  b.g.aux2 = up;
  b.g.ld_aux2 = ld_out;
  b.g.aux2_rows = rows;
  b.epi = moe::EPI_SWIGLU;
  b.op = GemmOperands{x, rows, hidden, ld_x, 0, w1, hidden, total_width, total_width, 1,
                      pick_bn(tile_n, 0), 0};
  b.op.pair = 1;
  b.op.grid = pick_ctas(tile_n);
  return b;
}

Built build_down(const void* inter, int64_t rows, int64_t ld_inter, const void* w2,
                 int64_t hidden, int64_t total_width, const int32_t* tok_off,
                 const int32_t* w_off, const int32_t* tpe, int E, void* out, int64_t ld_out,
                 int tile_n, int* status) {
  if (!common_ok(rows, hidden, total_width, tok_off, w_off, E) || !inter || !w2 || !out ||
      ld_inter < 16 || ld_inter % 8 != 0 || ld_out < hidden)
    return bad(MOE_ERR_BAD_ARG);
  Built b{};
  b.g = base_desc(tok_off, tpe, w_off, E, hidden, status);
  b.g.m_src = moe::DIM_TOKENS;
  b.g.n_src = moe::DIM_CONST;
  b.g.k_src = moe::DIM_WIDTH;
  b.g.a_m_base = moe::BASE_TOK;
  b.g.b_k_base = moe::BASE_WOFF;
  b.g.d_m_base = moe::BASE_TOK;
  b.g.d = out;
  b.g.ldd = ld_out;
  b.g.d_rows = rows;
  b.epi = moe::EPI_STORE;
  b.op = GemmOperands{inter, rows, ld_inter, ld_inter, 0, w2, total_width, hidden, hidden, 1,
                      pick_bn(tile_n, hidden), 0};
  b.op.pair = pick_pair(tile_n);
  b.op.grid = pick_ctas(tile_n);
  return b;
}

Built build_up_dx(const void* grad_act, int64_t rows, int64_t ld_ga, const void* w1,
                  int64_t hidden, int64_t total_width, const int32_t* tok_off,
                  const int32_t* w_off, const int32_t* tpe, int E, void* grad_x, int64_t ld_gx,
                  int tile_n, int* status) {
  if (!common_ok(rows, hidden, total_width, tok_off, w_off, E) || !grad_act || !w1 || !grad_x ||
      ld_ga < 16 || ld_ga % 8 != 0 || ld_gx < hidden)
    return bad(MOE_ERR_BAD_ARG);
  Built b{};
  b.g = base_desc(tok_off, tpe, w_off, E, hidden, status);
  b.g.m_src = moe::DIM_TOKENS;
  b.g.n_src = moe::DIM_CONST;
  b.g.k_src = moe::DIM_WIDTH;
  b.g.a_m_base = moe::BASE_TOK;
  b.g.b_k_base = moe::BASE_WOFF;
  b.g.d_m_base = moe::BASE_TOK;
  b.g.d = grad_x;
  b.g.ldd = ld_gx;
  b.g.d_rows = rows;
  b.epi = moe::EPI_STORE;
  // B = w1 read K-major: rows are the hidden (N) index, columns the width (K)
  b.op = GemmOperands{grad_act, rows, ld_ga, ld_ga, 0, w1, hidden, total_width, total_width, 0,
                      pick_bn(tile_n, hidden), 0};
  b.op.pair = pick_pair(tile_n);
  b.op.grid = pick_ctas(tile_n);
  return b;
}

Built build_up_dw(const void* x, int64_t rows, int64_t ld_x, const void* grad_act, int64_t ld_ga,
                  int64_t hidden, int64_t total_width, const int32_t* tok_off,
                  const int32_t* w_off, int E, void* grad_w1, int tile_n, int* status) {
  if (!common_ok(rows, hidden, total_width, tok_off, w_off, E) || !x || !grad_act || !grad_w1 ||
      ld_x < hidden || ld_ga < 16 || ld_ga % 8 != 0)
    return bad(MOE_ERR_BAD_ARG);
  Built b{};
  b.g = base_desc(tok_off, nullptr, w_off, E, hidden, status);
  b.g.m_src = moe::DIM_CONST;
  b.g.n_src = moe::DIM_WIDTH;
  b.g.k_src = moe::DIM_TOKENS;
  b.g.a_k_base = moe::BASE_TOK;
  b.g.b_k_base = moe::BASE_TOK;
  b.g.d_n_base = moe::BASE_WOFF;
  b.g.d = grad_w1;
  b.g.ldd = total_width;
  b.g.d_rows = hidden;
  b.epi = moe::EPI_STORE;
  b.op = GemmOperands{x, rows, hidden, ld_x, 1, grad_act, rows, ld_ga, ld_ga, 1,
                      pick_bn(tile_n, 0), 0};
  b.op.pair = pick_pair(tile_n);
  b.op.grid = pick_ctas(tile_n);
  return b;
}

Built build_down_dinter(const void* grad_y, int64_t rows, int64_t ld_gy, const void* w2,
                        int64_t hidden, int64_t total_width, const int32_t* tok_off,
                        const int32_t* w_off, const int32_t* tpe, int E, const void* pre_act,
                        int64_t ld_pre, void* out, int64_t ld_out, int tile_n, int* status) {
  if (!common_ok(rows, hidden, total_width, tok_off, w_off, E) || !grad_y || !w2 || !out ||
      ld_gy < hidden || ld_out < 16 || ld_out % 8 != 0 ||
      (pre_act && (ld_pre < 16 || ld_pre % 8 != 0)))
    return bad(MOE_ERR_BAD_ARG);
  Built b{};
  b.g = base_desc(tok_off, tpe, w_off, E, hidden, status);
  b.g.m_src = moe::DIM_TOKENS;
  b.g.n_src = moe::DIM_WIDTH;
  b.g.k_src = moe::DIM_CONST;
  b.g.a_m_base = moe::BASE_TOK;
  b.g.b_n_base = moe::BASE_WOFF;
  b.g.d_m_base = moe::BASE_TOK;
  b.g.d = out;
  b.g.ldd = ld_out;
  b.g.d_rows = rows;
  b.g.aux = const_cast<void*>(pre_act);
  b.g.ld_aux = ld_pre;
  b.g.aux_rows = rows;
  b.epi = pre_act ? moe::EPI_DACT : moe::EPI_STORE;
  // B = w2 read K-major: rows are the width (N) index, columns the hidden (K)
  b.op = GemmOperands{grad_y, rows, hidden, ld_gy, 0, w2, total_width, hidden, hidden, 0,
                      pick_bn(tile_n, 0), 0};
  b.op.pair = pick_pair(tile_n);
  b.op.grid = pick_ctas(tile_n);
  return b;
}

Built build_down_dw(const void* inter, int64_t rows, int64_t ld_inter, const void* grad_y,
                    int64_t ld_gy, int64_t hidden, int64_t total_width, const int32_t* tok_off,
                    const int32_t* w_off, int E, void* grad_w2, int tile_n, int* status) {
  if (!common_ok(rows, hidden, total_width, tok_off, w_off, E) || !inter || !grad_y ||
      !grad_w2 || ld_inter < 16 || ld_inter % 8 != 0 || ld_gy < hidden)
    return bad(MOE_ERR_BAD_ARG);
  Built b{};
  b.g = base_desc(tok_off, nullptr, w_off, E, hidden, status);
  b.g.m_src = moe::DIM_WIDTH;
  b.g.n_src = moe::DIM_CONST;
  b.g.k_src = moe::DIM_TOKENS;
  b.g.a_k_base = moe::BASE_TOK;
  b.g.b_k_base = moe::BASE_TOK;
  b.g.d_m_base = moe::BASE_WOFF;
  b.g.d = grad_w2;
  b.g.ldd = hidden;
  b.g.d_rows = total_width;
  b.epi = moe::EPI_STORE;
  b.op = GemmOperands{inter, rows, ld_inter, ld_inter, 1, grad_y, rows, hidden, ld_gy, 1,
                      pick_bn(tile_n, hidden), 0};
  b.op.pair = pick_pair(tile_n);
  b.op.grid = pick_ctas(tile_n);
  return b;
}

int run1(const Built& b, int dtype, void* stream) {
  if (b.err) return b.err;
  if (!gemm_dtype_ok(dtype)) return MOE_ERR_UNSUPPORTED;
  return moe::run_grouped_gemm(b.op, b.g, b.epi, dtype, S(stream));
}

int run2(const Built& a, const Built& b, int dtype, void* stream) {
  if (a.err) return a.err;
  if (b.err) return b.err;
  if (!gemm_dtype_ok(dtype)) return MOE_ERR_UNSUPPORTED;
  const GemmOperands ops[2] = {a.op, b.op};
  const GroupedGemmDesc gs[2] = {a.g, b.g};
  const int epis[2] = {a.epi, b.epi};
  return moe::run_grouped_gemms(ops, gs, epis, 2, dtype, S(stream));
}

}  // namespace

extern "C" {

int moe_grouped_gemm_up(const void* x, int64_t rows, int64_t ld_x, const void* w1,
                        int64_t hidden, int64_t total_width,
                        const int32_t* expert_token_offsets,
                        const int32_t* expert_weight_offsets, const int32_t* tokens_per_expert,
                        int num_experts, int activation, void* out, void* pre_act,
                        int64_t ld_out, int dtype, int tile_n, int* status, void* stream) {
  return run1(build_up(x, rows, ld_x, w1, hidden, total_width, expert_token_offsets,
                       expert_weight_offsets, tokens_per_expert, num_experts, activation, out,
                       pre_act, ld_out, tile_n, status),
              dtype, stream);
}

int moe_grouped_gemm_up_swiglu(const void* x, int64_t rows, int64_t ld_x, const void* w1,
                               int64_t hidden, int64_t total_width,
                               const int32_t* expert_token_offsets,
                               const int32_t* expert_weight_offsets,
                               const int32_t* tokens_per_expert, int num_experts, void* out,
                               void* gate, void* up, int64_t ld_out, int dtype, int tile_n,
                               int* status, void* stream) {
  return run1(build_up_swiglu(x, rows, ld_x, w1, hidden, total_width, expert_token_offsets,
                              expert_weight_offsets, tokens_per_expert, num_experts, out, gate,
                              up, ld_out, tile_n, status),
              dtype, stream);
}

int moe_swiglu_grad(const void* grad_out, const void* gate, const void* up, int64_t rows,
                    int64_t ld, const int32_t* expert_token_offsets,
                    const int32_t* expert_weight_offsets, int num_experts, void* grad_act,
                    int64_t ld_act, int dtype, void* stream) {
  if (rows < 0 || ld < 1 || ld_act < 1 || num_experts < 1 || num_experts > moe::kMaxGroups)
    return MOE_ERR_BAD_ARG;
  if (rows > 0 && (!grad_out || !gate || !up || !grad_act || !expert_token_offsets ||
                   !expert_weight_offsets))
    return MOE_ERR_BAD_ARG;
  return moe::swiglu_grad(grad_out, gate, up, rows, ld, expert_token_offsets,
                          expert_weight_offsets, num_experts, grad_act, ld_act, dtype, S(stream));
}

int64_t moe_up_down_dep_words(int64_t rows, int num_experts) {
  if (rows < 0 || num_experts < 1) return 0;
  return 2 * (rows / 128 + num_experts + 1);
}

int moe_grouped_gemm_up_down(const void* x, int64_t rows, int64_t ld_x, const void* w1,
                             const void* w2, int64_t hidden, int64_t total_width,
                             const int32_t* expert_token_offsets,
                             const int32_t* expert_weight_offsets,
                             const int32_t* tokens_per_expert, int num_experts, void* inter,
                             void* pre_act, int64_t ld_inter, void* out, int64_t ld_out,
                             int32_t* dep, int64_t dep_words, int dtype, int tile_n_width,
                             int tile_n_hidden, int* status, void* stream) {
  if (!dep || dep_words < moe_up_down_dep_words(rows, num_experts)) return MOE_ERR_BAD_ARG;
  Built up = build_up(x, rows, ld_x, w1, hidden, total_width, expert_token_offsets,
                      expert_weight_offsets, tokens_per_expert, num_experts,
                      MOE_ACT_RELU_SQUARED, inter, pre_act, ld_inter, tile_n_width, status);
  Built down = build_down(inter, rows, ld_inter, w2, hidden, total_width, expert_token_offsets,
                          expert_weight_offsets, tokens_per_expert, num_experts, out, ld_out,
                          tile_n_hidden, status);
  const int half = static_cast<int>(dep_words / 2);
  up.g.dep = dep;
  up.g.dep_len = half;
  up.g.dep_role = 1;
  down.g.dep = dep;
  down.g.dep_len = half;
  down.g.dep_role = 2;
  return run2(up, down, dtype, stream);
}

int moe_grouped_gemm_down(const void* inter, int64_t rows, int64_t ld_inter, const void* w2,
                          int64_t hidden, int64_t total_width,
                          const int32_t* expert_token_offsets,
                          const int32_t* expert_weight_offsets,
                          const int32_t* tokens_per_expert, int num_experts, void* out,
                          int64_t ld_out, int dtype, int tile_n, int* status, void* stream) {
  return run1(build_down(inter, rows, ld_inter, w2, hidden, total_width, expert_token_offsets,
                         expert_weight_offsets, tokens_per_expert, num_experts, out, ld_out,
                         tile_n, status),
              dtype, stream);
}

int moe_grouped_gemm_up_dx(const void* grad_act, int64_t rows, int64_t ld_grad_act,
                           const void* w1, int64_t hidden, int64_t total_width,
                           const int32_t* expert_token_offsets,
                           const int32_t* expert_weight_offsets,
                           const int32_t* tokens_per_expert, int num_experts, void* grad_x,
                           int64_t ld_grad_x, int dtype, int tile_n, int* status, void* stream) {
  return run1(build_up_dx(grad_act, rows, ld_grad_act, w1, hidden, total_width,
                          expert_token_offsets, expert_weight_offsets, tokens_per_expert,
                          num_experts, grad_x, ld_grad_x, tile_n, status),
              dtype, stream);
}

int moe_grouped_gemm_up_dw(const void* x, int64_t rows, int64_t ld_x, const void* grad_act,
                           int64_t ld_grad_act, int64_t hidden, int64_t total_width,
                           const int32_t* expert_token_offsets,
                           const int32_t* expert_weight_offsets, int num_experts,
                           void* grad_w1, int dtype, int tile_n, int* status, void* stream) {
  return run1(build_up_dw(x, rows, ld_x, grad_act, ld_grad_act, hidden, total_width,
                          expert_token_offsets, expert_weight_offsets, num_experts, grad_w1,
                          tile_n, status),
              dtype, stream);
}

int moe_grouped_gemm_down_dinter(const void* grad_y, int64_t rows, int64_t ld_grad_y,
                                 const void* w2, int64_t hidden, int64_t total_width,
                                 const int32_t* expert_token_offsets,
                                 const int32_t* expert_weight_offsets,
                                 const int32_t* tokens_per_expert, int num_experts,
                                 const void* pre_act, int64_t ld_pre, void* out, int64_t ld_out,
                                 int dtype, int tile_n, int* status, void* stream) {
  return run1(build_down_dinter(grad_y, rows, ld_grad_y, w2, hidden, total_width,
                                expert_token_offsets, expert_weight_offsets, tokens_per_expert,
                                num_experts, pre_act, ld_pre, out, ld_out, tile_n, status),
              dtype, stream);
}

int moe_grouped_gemm_down_dw(const void* inter, int64_t rows, int64_t ld_inter,
                             const void* grad_y, int64_t ld_grad_y, int64_t hidden,
                             int64_t total_width, const int32_t* expert_token_offsets,
                             const int32_t* expert_weight_offsets, int num_experts,
                             void* grad_w2, int dtype, int tile_n, int* status, void* stream) {
  return run1(build_down_dw(inter, rows, ld_inter, grad_y, ld_grad_y, hidden, total_width,
                            expert_token_offsets, expert_weight_offsets, num_experts, grad_w2,
                            tile_n, status),
              dtype, stream);
}

int moe_grouped_gemm_down_backward(const void* grad_y, int64_t rows, int64_t ld_grad_y,
                                   const void* inter, int64_t ld_inter, const void* w2,
                                   int64_t hidden, int64_t total_width,
                                   const int32_t* expert_token_offsets,
                                   const int32_t* expert_weight_offsets,
                                   const int32_t* tokens_per_expert, int num_experts,
                                   const void* pre_act, int64_t ld_pre, void* grad_inter,
                                   int64_t ld_grad_inter, void* grad_w2, int dtype,
                                   int tile_n_width, int tile_n_hidden, int* status,
                                   void* stream) {
  return run2(build_down_dinter(grad_y, rows, ld_grad_y, w2, hidden, total_width,
                                expert_token_offsets, expert_weight_offsets, tokens_per_expert,
                                num_experts, pre_act, ld_pre, grad_inter, ld_grad_inter,
                                tile_n_width, status),
              build_down_dw(inter, rows, ld_inter, grad_y, ld_grad_y, hidden, total_width,
                            expert_token_offsets, expert_weight_offsets, num_experts, grad_w2,
                            tile_n_hidden, status),
              dtype, stream);
}

int moe_grouped_gemm_up_backward(const void* grad_act, int64_t rows, int64_t ld_grad_act,
                                 const void* x, int64_t ld_x, const void* w1, int64_t hidden,
                                 int64_t total_width, const int32_t* expert_token_offsets,
                                 const int32_t* expert_weight_offsets,
                                 const int32_t* tokens_per_expert, int num_experts,
                                 void* grad_x, int64_t ld_grad_x, void* grad_w1, int dtype,
                                 int tile_n_width, int tile_n_hidden, int* status,
                                 void* stream) {
  return run2(build_up_dx(grad_act, rows, ld_grad_act, w1, hidden, total_width,
                          expert_token_offsets, expert_weight_offsets, tokens_per_expert,
                          num_experts, grad_x, ld_grad_x, tile_n_hidden, status),
              build_up_dw(x, rows, ld_x, grad_act, ld_grad_act, hidden, total_width,
                          expert_token_offsets, expert_weight_offsets, num_experts, grad_w1,
                          tile_n_width, status),
              dtype, stream);
}

}  // extern "C"
