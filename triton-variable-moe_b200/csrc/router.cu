// Top-k expert choice and weight renormalisation for the router output.
//
// Restates triton_moe/moe.py:168-182 after the sigmoid: torch.topk(probs, k)
// (values in descending order, indices beside them), then, when normalising,
// w / (sum_k w + 1e-20) in fp32, cast to the storage dtype.  Ties between
// equal probabilities go to the lower expert index.  One warp per token: each
// lane holds ceil(E/32) probabilities in registers and k rounds of a warp
// arg-max pick the experts, so the whole choice is one pass over [T, E].
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "moe_internal.h"

namespace moe {
namespace {

template <typename T>
__device__ __forceinline__ T from_float(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_float<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ float from_float<float>(float v) {
  return v;
}

constexpr int kTopkMax = 32;  // largest top_k handled (one value per lane)

// (value, index) ordering of torch.topk on distinct values; equal values go to
// the lower index.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

template <typename TW, int NV>
__global__ void __launch_bounds__(256)
    topk_kernel(const float* __restrict__ probs, long long T, int E, int k, int normalize,
                TW* __restrict__ w_out, int32_t* __restrict__ sel_out) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long t = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       t < T; t += warps) {
    const float* row = probs + t * E;
    float v[NV];
    unsigned used = 0;  // bit j: this lane's value j was already chosen
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int e = j * 32 + lane;
      v[j] = e < E ? row[e] : 0.f;
    }
    float my_val = 0.f;  // lane s keeps the s-th chosen value
    int my_idx = 0;
    for (int s = 0; s < k; ++s) {
      float bv = -__int_as_float(0x7f800000);  // -inf
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int e = j * 32 + lane;
        if (e < E && !((used >> j) & 1u) && better(v[j], e, bv, bi)) {
          bv = v[j];
          bi = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (bi != 0x7fffffff && (bi & 31) == lane) used |= 1u << (bi >> 5);
      if (lane == s) {
        my_val = bv;
        my_idx = bi;
      }
    }
    float denom = 1.f;
    if (normalize) {
      float sum = 0.f;  // sequential in rank order
      for (int s = 0; s < k; ++s) sum += __shfl_sync(0xffffffffu, my_val, s);
      denom = sum + 1e-20f;
    }
    if (lane < k) {
      const float w = normalize ? my_val / denom : my_val;
      w_out[t * k + lane] = from_float<TW>(w);
      sel_out[t * k + lane] = my_idx;
    }
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename TW, int NV>
int launch_topk(const float* probs, long long T, int E, int k, int norm, void* w, int32_t* sel,
                cudaStream_t st) {
  long long blocks = (T + 7) / 8;
  const long long cap = static_cast<long long>(num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, topk_kernel<TW, NV>, probs, T, E, k, norm, static_cast<TW*>(w),
                         sel) != cudaSuccess)
    return kStatusCuda;
  return cudaPeekAtLastError() == cudaSuccess ? kStatusOk : kStatusCuda;
}

template <typename TW>
int topk_dispatch(const float* probs, long long T, int E, int k, int norm, void* w, int32_t* sel,
                  cudaStream_t st) {
  if (E <= 32) return launch_topk<TW, 1>(probs, T, E, k, norm, w, sel, st);
  if (E <= 64) return launch_topk<TW, 2>(probs, T, E, k, norm, w, sel, st);
  if (E <= 128) return launch_topk<TW, 4>(probs, T, E, k, norm, w, sel, st);
  return launch_topk<TW, 8>(probs, T, E, k, norm, w, sel, st);
}

}  // namespace

int router_topk(const float* probs, long long T, int E, int k, int norm, void* w, int w_dtype,
                int32_t* sel, cudaStream_t st) {
  if (T < 0 || E <= 0 || E > 256 || k <= 0 || k > E || k > kTopkMax) return kStatusBadArg;
  if (T == 0) return kStatusOk;
  if (!probs || !w || !sel) return kStatusBadArg;
  if (w_dtype == 0) return topk_dispatch<__nv_bfloat16>(probs, T, E, k, norm, w, sel, st);
  if (w_dtype == 1) return topk_dispatch<__half>(probs, T, E, k, norm, w, sel, st);
  if (w_dtype == 2) return topk_dispatch<float>(probs, T, E, k, norm, w, sel, st);
  return kStatusUnsupported;
}

}  // namespace moe

// ---- fused router head and auxiliary losses ------------------------------------
// router_head: from the router logits [T, E] (storage dtype L) computes, in one
// pass with one warp per token,
//   probs = sigmoid(float(logits))                       (moe.py:168)
//   top-k choice and renormalised weights                (moe.py:170-179)
//   lse_t = logsumexp(logits_t) with the rounding chain of torch's logsumexp in
//           dtype L: max, x - max, exp, sum (fp32 accumulate), log, + max
//   per-block partial sums of probs[:, e], lse_t^2 (rounded to L) and
//   sum_e probs[t, e] * widths_norm[e]                   (moe.py:253-268)
// aux_finalize (one block) reduces the partials in a fixed order and forms
// router_z_loss, load_balance_loss, compute_loss and f_i (moe.py:253-303).
namespace moe {
namespace {

template <typename T>
__device__ __forceinline__ float to_float(T v);
template <>
__device__ __forceinline__ float to_float<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_float<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_float<float>(float v) {
  return v;
}
template <typename T>
__device__ __forceinline__ float rnd(float v) {
  return to_float<T>(from_float<T>(v));
}

constexpr int kHeadWarps = 8;

// One block of 256 threads.  losses[0] = router_z_loss (value rounded to L),
// losses[1] = load_balance_loss, losses[2] = compute_loss; f_i in TF; p_i
// (fp32) kept for the backward.  lb = sum_e coef[e] * f_i[e] * p_i[e].
// partials: per block [E probability sums, z sum, compute sum (, E selection
// counts)] with the given stride; the expert counts come from tpe when it is
// given, else from the partials' count sums.
template <typename L, typename TF>
__device__ void aux_finalize_block(const float* partials, int nblocks, int stride, int E,
                                   long long T, const int32_t* tpe, const float* lb_coef,
                                   float* losses, TF* f_i, float* p_i, L* z_out) {
  __shared__ float s_part[256];
  __shared__ float s_col[2 * 256 + 2];  // column sums over the blocks
  __shared__ float s_red[256];
  __shared__ long long s_cnt[256];
  const int tid = threadIdx.x;
  const bool counts_in_partials = tpe == nullptr;
  // Column sums over the blocks, one pass: G threads per column, each keeping
  // up to 16 independent loads in flight; the G partial sums are then added
  // in a fixed order (the result does not depend on timing).
  const int C = counts_in_partials ? 2 * E + 2 : E + 2;
  const int G = max(1, 256 / C);
  for (int c0 = 0; c0 < C; c0 += 256 / G) {
    const int c = c0 + tid / G, g = tid % G;
    float v = 0.f;
    if (c < C && tid / G < 256 / G) {
      float acc[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = 0.f;
      int b = g;
      for (; b + 15 * G < nblocks; b += 16 * G) {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          acc[i] += __ldcg(partials + static_cast<long long>(b + i * G) * stride + c);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i)  // the last < 16 blocks of this thread
        if (b + i * G < nblocks)
          acc[i] += __ldcg(partials + static_cast<long long>(b + i * G) * stride + c);
#pragma unroll
      for (int w = 8; w > 0; w >>= 1)
#pragma unroll
        for (int i = 0; i < w; ++i) acc[i] += acc[i + w];
      v = acc[0];
    }
    s_part[tid] = v;
    __syncthreads();
    if (g == 0 && c < C && tid / G < 256 / G) {
      float tot = 0.f;
      for (int q = 0; q < G; ++q) tot += s_part[tid + q];
      s_col[c] = tot;
    }
    __syncthreads();
  }
  const float* s_pe = s_col;          // per-expert probability sums
  const float* s_ce = s_col + E + 2;  // per-expert selection counts
  long long cnt = 0;
  for (int e = tid; e < E; e += blockDim.x)
    cnt += counts_in_partials ? static_cast<long long>(s_ce[e]) : tpe[e];
  s_cnt[tid] = cnt;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (tid < o) s_cnt[tid] += s_cnt[tid + o];
    __syncthreads();
  }
  const float zsum = s_col[E], csum = s_col[E + 1];
  const float total = static_cast<float>(s_cnt[0]);
  const float invT = 1.0f / static_cast<float>(T);
  __syncthreads();
  float lb = 0.f;
  for (int e = tid; e < E; e += blockDim.x) {
    const float pe = s_pe[e] * invT;
    p_i[e] = pe;
    const float ce = counts_in_partials ? s_ce[e] : static_cast<float>(tpe[e]);
    const TF f = from_float<TF>(ce / total);
    f_i[e] = f;
    lb += lb_coef[e] * to_float<TF>(f) * pe;
  }
  s_red[tid] = lb;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (tid < o) s_red[tid] += s_red[tid + o];
    __syncthreads();
  }
  if (tid == 0) {
    losses[0] = rnd<L>(zsum * invT);
    if (z_out != nullptr) *z_out = from_float<L>(zsum * invT);
    losses[1] = s_red[0];
    losses[2] = csum * invT;
  }
}

template <typename L, typename TF>
__global__ void __launch_bounds__(256)
    aux_finalize_kernel(const float* __restrict__ partials, int nblocks, int stride, int E,
                        long long T, const int32_t* __restrict__ tpe,
                        const float* __restrict__ lb_coef, float* __restrict__ losses,
                        TF* __restrict__ f_i, float* __restrict__ p_i, L* __restrict__ z_out) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  aux_finalize_block<L, TF>(partials, nblocks, stride, E, T, tpe, lb_coef, losses, f_i, p_i,
                            z_out);
}

// Auxiliary-loss outputs of the fused head (all null: partials only).
template <typename L, typename TF>
struct HeadLosses {
  const float* lb_coef;
  float* losses;
  TF* f_i;
  float* p_i;
  L* z_out;
  unsigned* ticket;  // zero before the launch; the last block returns it to zero
};

// With loss outputs given, every block also counts its tokens' selected
// experts, and the last block to finish (a ticket taken after the block's
// partials are published) reduces all partials into the losses: the loss
// finalisation costs no extra launch.
// Layout: a token is handled by a group of G lanes (a power of two), each lane
// holding EPL = 8 of its experts in registers (expert e in lane e / 8 of the
// group); a warp works on 32 / G tokens at once.  Reductions over a token's
// experts run over the lane's 8 slots and then log2(G) xor-shuffles inside the
// group, so the dependent shuffle chain per token is short and each warp has
// 32 / G independent tokens in flight; the next step's logits are loaded
// while the current step is processed.
template <typename L, typename TW, int G>
__global__ void __launch_bounds__(kHeadWarps * 32)
    router_head_kernel(const L* __restrict__ logits, long long T, int E, int k, int normalize,
                       const float* __restrict__ widths_norm, float* __restrict__ probs,
                       TW* __restrict__ w_out, int32_t* __restrict__ sel_out,
                       float* __restrict__ lse_out, float* __restrict__ partials,
                       HeadLosses<L, TW> fin) {
  constexpr int EPL = 8;
  constexpr int TPW = 32 / G;  // tokens per warp step
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float s_p[kHeadWarps][G * EPL];
  __shared__ int s_n[kHeadWarps][G * EPL];
  __shared__ float s_z[kHeadWarps], s_c[kHeadWarps];
  __shared__ unsigned s_ticket;
  const bool fused = fin.losses != nullptr;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int g = lane % G;   // lane within the token's group
  const int tg = lane / G;  // token within the warp step
  const int e0 = g * EPL;   // this lane's first expert
  const float NEG_INF = -__int_as_float(0x7f800000);
  float acc_p[EPL], wn[EPL];
  int cnt[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    acc_p[i] = 0.f;
    cnt[i] = 0;
    wn[i] = e0 + i < E ? widths_norm[e0 + i] : 0.f;
  }
  float acc_z = 0.f, acc_c = 0.f;
  const long long step = static_cast<long long>(gridDim.x) * kHeadWarps * TPW;
  const long long first = (static_cast<long long>(blockIdx.x) * kHeadWarps + wid) * TPW;
  auto load = [&](long long tb, float (&x)[EPL]) {
    const long long t = tb + tg;
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      x[i] = (t < T && e0 + i < E) ? to_float<L>(logits[t * E + e0 + i]) : NEG_INF;
  };
  // arg-max over this token's experts not yet chosen (lower index on ties)
  auto group_best = [&](const float (&p)[EPL], unsigned used, float& bv, int& bi) {
    bv = NEG_INF;
    bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (e0 + i < E && !((used >> i) & 1u) && better(p[i], e0 + i, bv, bi)) {
        bv = p[i];
        bi = e0 + i;
      }
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
  };
  float x[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) x[i] = NEG_INF;
  if (first < T) load(first, x);
  for (long long tb = first; tb < T; tb += step) {  // warp-uniform loop
    const long long t = tb + tg;
    const bool valid = t < T;
    float xn[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) xn[i] = NEG_INF;
    if (tb + step < T) load(tb + step, xn);  // next step's logits in flight
    float m = NEG_INF;
#pragma unroll
    for (int i = 0; i < EPL; ++i) m = fmaxf(m, x[i]);
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float mm = isinf(m) ? 0.f : m;
    float s = 0.f, c = 0.f, p[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      if (valid && e0 + i < E) {
        s += rnd<L>(expf(rnd<L>(x[i] - mm)));
        p[i] = 1.0f / (1.0f + expf(-x[i]));
        acc_p[i] += p[i];
        c += p[i] * wn[i];
      } else {
        p[i] = NEG_INF;
      }
    }
    if (valid && e0 < E) {
      float* prow = probs + t * E + e0;
      if ((E & 7) == 0) {
        reinterpret_cast<float4*>(prow)[0] = make_float4(p[0], p[1], p[2], p[3]);
        reinterpret_cast<float4*>(prow)[1] = make_float4(p[4], p[5], p[6], p[7]);
      } else {
#pragma unroll
        for (int i = 0; i < EPL; ++i)
          if (e0 + i < E) prow[i] = p[i];
      }
    }
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) {
      s += __shfl_xor_sync(0xffffffffu, s, o);
      c += __shfl_xor_sync(0xffffffffu, c, o);
    }
    const float lse = rnd<L>(rnd<L>(logf(rnd<L>(s))) + mm);
    if (valid && g == 0) {
      lse_out[t] = lse;
      acc_z += rnd<L>(lse * lse);
      acc_c += c;
    }
    // top-k (torch.topk order); with renormalisation the k rounds run twice:
    // first for the denominator (summed in rank order), then for the writes
    float denom = 1.f;
    if (normalize) {
      unsigned used = 0;
      float sum = 0.f;
      for (int r = 0; r < k; ++r) {
        float bv;
        int bi;
        group_best(p, used, bv, bi);
        sum += bv;
        if (bi >= e0 && bi < e0 + EPL) used |= 1u << (bi - e0);
      }
      denom = sum + 1e-20f;
    }
    unsigned used = 0;
    for (int r = 0; r < k; ++r) {
      float bv;
      int bi;
      group_best(p, used, bv, bi);
      if (bi >= e0 && bi < e0 + EPL) {
        used |= 1u << (bi - e0);
        if (valid) {
#pragma unroll
          for (int i = 0; i < EPL; ++i)
            if (bi == e0 + i) ++cnt[i];
        }
      }
      if (valid && g == 0) {
        w_out[t * k + r] = from_float<TW>(normalize ? bv / denom : bv);
        sel_out[t * k + r] = bi;
      }
    }
#pragma unroll
    for (int i = 0; i < EPL; ++i) x[i] = xn[i];
  }
  // block partials: per-expert probability sums (and selection counts), then
  // the z and compute-loss sums; fixed reduction order throughout
#pragma unroll
  for (int i = 0; i < EPL; ++i)
#pragma unroll
    for (int o = G; o < 32; o <<= 1) {
      acc_p[i] += __shfl_xor_sync(0xffffffffu, acc_p[i], o);
      cnt[i] += __shfl_xor_sync(0xffffffffu, cnt[i], o);
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc_z += __shfl_xor_sync(0xffffffffu, acc_z, o);
    acc_c += __shfl_xor_sync(0xffffffffu, acc_c, o);
  }
  if (lane < G) {
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      s_p[wid][lane * EPL + i] = acc_p[i];
      s_n[wid][lane * EPL + i] = cnt[i];
    }
  }
  if (lane == 0) {
    s_z[wid] = acc_z;
    s_c[wid] = acc_c;
  }
  __syncthreads();
  const int stride = 2 * E + 2;
  float* out = partials + static_cast<long long>(blockIdx.x) * stride;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    float v = 0.f;
    int n = 0;
    for (int w = 0; w < kHeadWarps; ++w) {
      v += s_p[w][e];
      n += s_n[w][e];
    }
    out[e] = v;
    out[E + 2 + e] = static_cast<float>(n);
  }
  if (threadIdx.x == 0) {
    float z = 0.f, cc = 0.f;
    for (int w = 0; w < kHeadWarps; ++w) {
      z += s_z[w];
      cc += s_c[w];
    }
    out[E] = z;
    out[E + 1] = cc;
  }
  if (fused) {
    // publish this block's partials, then take a ticket; the last block sums
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_ticket = atomicAdd(fin.ticket, 1u);
    __syncthreads();
    if (s_ticket == gridDim.x - 1) {
      __threadfence();
      aux_finalize_block<L, TW>(partials, gridDim.x, stride, E, T, nullptr, fin.lb_coef,
                                fin.losses, fin.f_i, fin.p_i, fin.z_out);
      if (threadIdx.x == 0) atomicExch(fin.ticket, 0u);
    }
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Loss outputs of a fused head launch (null losses: partials only).
struct LossArgs {
  const float* lb_coef;
  float* losses;
  void* f_i;  // weights dtype
  float* p_i;
  void* z_out;  // logits dtype
  unsigned* ticket;
};

template <typename L, typename TW, int G>
int launch_head(const void* logits, long long T, int E, int k, int norm, const float* wn,
                float* probs, void* w, int32_t* sel, float* lse, float* part, int nblocks,
                const LossArgs& la, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nblocks);
  cfg.blockDim = dim3(kHeadWarps * 32);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  HeadLosses<L, TW> fin{la.lb_coef, la.losses, static_cast<TW*>(la.f_i), la.p_i,
                        static_cast<L*>(la.z_out), la.ticket};
  if (cudaLaunchKernelEx(&cfg, router_head_kernel<L, TW, G>, static_cast<const L*>(logits), T, E,
                         k, norm, wn, probs, static_cast<TW*>(w), sel, lse, part, fin) !=
      cudaSuccess)
    return kStatusCuda;
  return cudaPeekAtLastError() == cudaSuccess ? kStatusOk : kStatusCuda;
}

template <typename L, typename TW>
int head_nv(const void* logits, long long T, int E, int k, int norm, const float* wn, float* probs,
            void* w, int32_t* sel, float* lse, float* part, int nb, const LossArgs& la,
            cudaStream_t st) {
  // lanes per token at 8 experts per lane
  if (E <= 8) return launch_head<L, TW, 1>(logits, T, E, k, norm, wn, probs, w, sel, lse, part, nb, la, st);
  if (E <= 16) return launch_head<L, TW, 2>(logits, T, E, k, norm, wn, probs, w, sel, lse, part, nb, la, st);
  if (E <= 32) return launch_head<L, TW, 4>(logits, T, E, k, norm, wn, probs, w, sel, lse, part, nb, la, st);
  if (E <= 64) return launch_head<L, TW, 8>(logits, T, E, k, norm, wn, probs, w, sel, lse, part, nb, la, st);
  if (E <= 128) return launch_head<L, TW, 16>(logits, T, E, k, norm, wn, probs, w, sel, lse, part, nb, la, st);
  return launch_head<L, TW, 32>(logits, T, E, k, norm, wn, probs, w, sel, lse, part, nb, la, st);
}

template <typename L>
int head_tw(const void* logits, long long T, int E, int k, int norm, const float* wn, float* probs,
            void* w, int w_dtype, int32_t* sel, float* lse, float* part, int nb,
            const LossArgs& la, cudaStream_t st) {
  if (w_dtype == 0) return head_nv<L, __nv_bfloat16>(logits, T, E, k, norm, wn, probs, w, sel, lse, part, nb, la, st);
  if (w_dtype == 1) return head_nv<L, __half>(logits, T, E, k, norm, wn, probs, w, sel, lse, part, nb, la, st);
  if (w_dtype == 2) return head_nv<L, float>(logits, T, E, k, norm, wn, probs, w, sel, lse, part, nb, la, st);
  return kStatusUnsupported;
}

template <typename L, typename TF>
int launch_finalize(const float* part, int nb, int E, long long T, const int32_t* tpe,
                    const float* coef, float* losses, void* f_i, float* p_i, void* z_out,
                    cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, aux_finalize_kernel<L, TF>, part, nb, 2 * E + 2, E, T, tpe, coef,
                         losses, static_cast<TF*>(f_i), p_i, static_cast<L*>(z_out)) !=
      cudaSuccess)
    return kStatusCuda;
  return cudaPeekAtLastError() == cudaSuccess ? kStatusOk : kStatusCuda;
}

template <typename L>
int finalize_tf(const float* part, int nb, int E, long long T, const int32_t* tpe,
                const float* coef, float* losses, void* f_i, int f_dtype, float* p_i, void* z_out,
                cudaStream_t st) {
  if (f_dtype == 0) return launch_finalize<L, __nv_bfloat16>(part, nb, E, T, tpe, coef, losses, f_i, p_i, z_out, st);
  if (f_dtype == 1) return launch_finalize<L, __half>(part, nb, E, T, tpe, coef, losses, f_i, p_i, z_out, st);
  if (f_dtype == 2) return launch_finalize<L, float>(part, nb, E, T, tpe, coef, losses, f_i, p_i, z_out, st);
  return kStatusUnsupported;
}

}  // namespace

int router_head_blocks(long long T) {
  long long b = (T + 4 * kHeadWarps - 1) / (4 * kHeadWarps);
  const long long cap = static_cast<long long>(num_sms());
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return static_cast<int>(b);
}

int router_head(const void* logits, int l_dtype, long long T, int E, int k, int norm,
                const float* widths_norm, float* probs, void* w, int w_dtype, int32_t* sel,
                float* lse, float* partials, int nblocks, const float* lb_coef, float* losses,
                void* f_i, float* p_i, void* z_out, unsigned* ticket, cudaStream_t st) {
  if (T < 0 || E <= 0 || E > 256 || k <= 0 || k > E || k > kTopkMax) return kStatusBadArg;
  if (nblocks != router_head_blocks(T)) return kStatusBadArg;
  if (!logits || !widths_norm || !probs || !w || !sel || !lse || !partials) return kStatusBadArg;
  if (losses != nullptr && (T == 0 || !lb_coef || !f_i || !p_i || !ticket)) return kStatusBadArg;
  const LossArgs la{lb_coef, losses, f_i, p_i, z_out, ticket};
  if (l_dtype == 0) return head_tw<__nv_bfloat16>(logits, T, E, k, norm, widths_norm, probs, w, w_dtype, sel, lse, partials, nblocks, la, st);
  if (l_dtype == 1) return head_tw<__half>(logits, T, E, k, norm, widths_norm, probs, w, w_dtype, sel, lse, partials, nblocks, la, st);
  if (l_dtype == 2) return head_tw<float>(logits, T, E, k, norm, widths_norm, probs, w, w_dtype, sel, lse, partials, nblocks, la, st);
  return kStatusUnsupported;
}

int aux_finalize(const float* partials, int nblocks, int E, long long T, const int32_t* tpe,
                 const float* lb_coef, int l_dtype, float* losses, void* f_i, int f_dtype,
                 float* p_i, void* z_out, cudaStream_t st) {
  if (E <= 0 || E > 256 || T <= 0 || nblocks <= 0) return kStatusBadArg;  // tpe may be null
  if (l_dtype == 0) return finalize_tf<__nv_bfloat16>(partials, nblocks, E, T, tpe, lb_coef, losses, f_i, f_dtype, p_i, z_out, st);
  if (l_dtype == 1) return finalize_tf<__half>(partials, nblocks, E, T, tpe, lb_coef, losses, f_i, f_dtype, p_i, z_out, st);
  if (l_dtype == 2) return finalize_tf<float>(partials, nblocks, E, T, tpe, lb_coef, losses, f_i, f_dtype, p_i, z_out, st);
  return kStatusUnsupported;
}

}  // namespace moe
