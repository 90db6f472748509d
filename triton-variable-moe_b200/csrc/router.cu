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

template <typename L, typename TW, int NV>
__global__ void __launch_bounds__(kHeadWarps * 32)
    router_head_kernel(const L* __restrict__ logits, long long T, int E, int k, int normalize,
                       const float* __restrict__ widths_norm, float* __restrict__ probs,
                       TW* __restrict__ w_out, int32_t* __restrict__ sel_out,
                       float* __restrict__ lse_out, float* __restrict__ partials) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float s_p[kHeadWarps][NV * 32];
  __shared__ float s_z[kHeadWarps], s_c[kHeadWarps];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const float NEG_INF = -__int_as_float(0x7f800000);
  float acc_p[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) acc_p[j] = 0.f;
  float acc_z = 0.f, acc_c = 0.f;
  float wn[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int e = j * 32 + lane;
    wn[j] = e < E ? widths_norm[e] : 0.f;
  }
  const long long warps = static_cast<long long>(gridDim.x) * kHeadWarps;
  for (long long t = static_cast<long long>(blockIdx.x) * kHeadWarps + wid; t < T; t += warps) {
    const L* row = logits + t * E;
    float x[NV], p[NV];
    float m = NEG_INF;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int e = j * 32 + lane;
      x[j] = e < E ? to_float<L>(row[e]) : NEG_INF;
      m = fmaxf(m, x[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float mm = isinf(m) ? 0.f : m;
    float s = 0.f;
    float c = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int e = j * 32 + lane;
      if (e < E) {
        s += rnd<L>(expf(rnd<L>(x[j] - mm)));
        p[j] = 1.0f / (1.0f + expf(-x[j]));
        probs[t * E + e] = p[j];
        acc_p[j] += p[j];
        c += p[j] * wn[j];
      } else {
        p[j] = 0.f;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s += __shfl_xor_sync(0xffffffffu, s, o);
      c += __shfl_xor_sync(0xffffffffu, c, o);
    }
    const float lse = rnd<L>(rnd<L>(logf(rnd<L>(s))) + mm);
    if (lane == 0) {
      lse_out[t] = lse;
      acc_z += rnd<L>(lse * lse);
      acc_c += c;
    }
    // top-k over probs (lower index on ties), renormalised weights
    unsigned used = 0;
    float my_val = 0.f;
    int my_idx = 0;
    for (int r = 0; r < k; ++r) {
      float bv = NEG_INF;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int e = j * 32 + lane;
        if (e < E && !((used >> j) & 1u) && better(p[j], e, bv, bi)) {
          bv = p[j];
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
      if (lane == r) {
        my_val = bv;
        my_idx = bi;
      }
    }
    float denom = 1.f;
    if (normalize) {
      float sum = 0.f;
      for (int r = 0; r < k; ++r) sum += __shfl_sync(0xffffffffu, my_val, r);
      denom = sum + 1e-20f;
    }
    if (lane < k) {
      w_out[t * k + lane] = from_float<TW>(normalize ? my_val / denom : my_val);
      sel_out[t * k + lane] = my_idx;
    }
  }
  // block partials: [E] probs sums, then z and compute-loss sums
#pragma unroll
  for (int j = 0; j < NV; ++j) s_p[wid][j * 32 + lane] = acc_p[j];
  if (lane == 0) {
    s_z[wid] = acc_z;
    s_c[wid] = acc_c;
  }
  __syncthreads();
  float* out = partials + static_cast<long long>(blockIdx.x) * (E + 2);
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    float v = 0.f;
    for (int w = 0; w < kHeadWarps; ++w) v += s_p[w][e];
    out[e] = v;
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
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// One block.  losses[0] = router_z_loss (value rounded to L), losses[1] =
// load_balance_loss, losses[2] = compute_loss; f_i in TF; p_i (fp32) kept for
// the backward.  lb = sum_e coef[e] * f_i[e] * p_i[e].
template <typename L, typename TF>
__global__ void __launch_bounds__(256)
    aux_finalize_kernel(const float* __restrict__ partials, int nblocks, int E, long long T,
                        const int32_t* __restrict__ tpe, const float* __restrict__ lb_coef,
                        float* __restrict__ losses, TF* __restrict__ f_i, float* __restrict__ p_i,
                        L* __restrict__ z_out) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float s_part[256];
  __shared__ float s_pe[256];
  __shared__ float s_red[256], s_red2[256];
  __shared__ long long s_cnt[256];
  const int tid = threadIdx.x;
  const int stride = E + 2;
  // per-expert sums of the block partials: threads (e, part) with parts = 256 / E
  const int parts = max(1, 256 / E);
  for (int e0 = 0; e0 < E; e0 += 256 / parts) {
    const int e = e0 + tid / parts;
    const int part = tid % parts;
    float v = 0.f;
    if (e < E && tid / parts < 256 / parts) {
      // four independent accumulators keep four loads in flight
      float v0 = 0.f, v1 = 0.f, v2 = 0.f, v3 = 0.f;
      int b = part;
      for (; b + 3 * parts < nblocks; b += 4 * parts) {
        v0 += partials[static_cast<long long>(b) * stride + e];
        v1 += partials[static_cast<long long>(b + parts) * stride + e];
        v2 += partials[static_cast<long long>(b + 2 * parts) * stride + e];
        v3 += partials[static_cast<long long>(b + 3 * parts) * stride + e];
      }
      for (; b < nblocks; b += parts) v0 += partials[static_cast<long long>(b) * stride + e];
      v = (v0 + v1) + (v2 + v3);
    }
    s_part[tid] = v;
    __syncthreads();
    if (part == 0 && e < E && tid / parts < 256 / parts) {
      float tot = 0.f;
      for (int q = 0; q < parts; ++q) tot += s_part[tid + q];
      s_pe[e] = tot;
    }
    __syncthreads();
  }
  // z-loss and compute-loss sums, assignment count
  float z = 0.f, c = 0.f;
  for (int b = tid; b < nblocks; b += blockDim.x) {
    z += partials[static_cast<long long>(b) * stride + E];
    c += partials[static_cast<long long>(b) * stride + E + 1];
  }
  long long cnt = 0;
  for (int e = tid; e < E; e += blockDim.x) cnt += tpe[e];
  s_red[tid] = z;
  s_red2[tid] = c;
  s_cnt[tid] = cnt;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (tid < o) {
      s_red[tid] += s_red[tid + o];
      s_red2[tid] += s_red2[tid + o];
      s_cnt[tid] += s_cnt[tid + o];
    }
    __syncthreads();
  }
  const float zsum = s_red[0], csum = s_red2[0];
  const float total = static_cast<float>(s_cnt[0]);
  const float invT = 1.0f / static_cast<float>(T);
  __syncthreads();
  float lb = 0.f;
  for (int e = tid; e < E; e += blockDim.x) {
    const float pe = s_pe[e] * invT;
    p_i[e] = pe;
    const TF f = from_float<TF>(static_cast<float>(tpe[e]) / total);
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

template <typename L, typename TW, int NV>
int launch_head(const void* logits, long long T, int E, int k, int norm, const float* wn,
                float* probs, void* w, int32_t* sel, float* lse, float* part, int nblocks,
                cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nblocks);
  cfg.blockDim = dim3(kHeadWarps * 32);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, router_head_kernel<L, TW, NV>, static_cast<const L*>(logits), T, E,
                         k, norm, wn, probs, static_cast<TW*>(w), sel, lse, part) != cudaSuccess)
    return kStatusCuda;
  return cudaPeekAtLastError() == cudaSuccess ? kStatusOk : kStatusCuda;
}

template <typename L, typename TW>
int head_nv(const void* logits, long long T, int E, int k, int norm, const float* wn, float* probs,
            void* w, int32_t* sel, float* lse, float* part, int nb, cudaStream_t st) {
  if (E <= 32) return launch_head<L, TW, 1>(logits, T, E, k, norm, wn, probs, w, sel, lse, part, nb, st);
  if (E <= 64) return launch_head<L, TW, 2>(logits, T, E, k, norm, wn, probs, w, sel, lse, part, nb, st);
  if (E <= 128) return launch_head<L, TW, 4>(logits, T, E, k, norm, wn, probs, w, sel, lse, part, nb, st);
  return launch_head<L, TW, 8>(logits, T, E, k, norm, wn, probs, w, sel, lse, part, nb, st);
}

template <typename L>
int head_tw(const void* logits, long long T, int E, int k, int norm, const float* wn, float* probs,
            void* w, int w_dtype, int32_t* sel, float* lse, float* part, int nb, cudaStream_t st) {
  if (w_dtype == 0) return head_nv<L, __nv_bfloat16>(logits, T, E, k, norm, wn, probs, w, sel, lse, part, nb, st);
  if (w_dtype == 1) return head_nv<L, __half>(logits, T, E, k, norm, wn, probs, w, sel, lse, part, nb, st);
  if (w_dtype == 2) return head_nv<L, float>(logits, T, E, k, norm, wn, probs, w, sel, lse, part, nb, st);
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
  if (cudaLaunchKernelEx(&cfg, aux_finalize_kernel<L, TF>, part, nb, E, T, tpe, coef, losses,
                         static_cast<TF*>(f_i), p_i, static_cast<L*>(z_out)) != cudaSuccess)
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
  long long b = (T + kHeadWarps - 1) / kHeadWarps;
  const long long cap = static_cast<long long>(num_sms()) * 2;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return static_cast<int>(b);
}

int router_head(const void* logits, int l_dtype, long long T, int E, int k, int norm,
                const float* widths_norm, float* probs, void* w, int w_dtype, int32_t* sel,
                float* lse, float* partials, int nblocks, cudaStream_t st) {
  if (T < 0 || E <= 0 || E > 256 || k <= 0 || k > E || k > kTopkMax) return kStatusBadArg;
  if (nblocks != router_head_blocks(T)) return kStatusBadArg;
  if (!logits || !widths_norm || !probs || !w || !sel || !lse || !partials) return kStatusBadArg;
  if (l_dtype == 0) return head_tw<__nv_bfloat16>(logits, T, E, k, norm, widths_norm, probs, w, w_dtype, sel, lse, partials, nblocks, st);
  if (l_dtype == 1) return head_tw<__half>(logits, T, E, k, norm, widths_norm, probs, w, w_dtype, sel, lse, partials, nblocks, st);
  if (l_dtype == 2) return head_tw<float>(logits, T, E, k, norm, widths_norm, probs, w, w_dtype, sel, lse, partials, nblocks, st);
  return kStatusUnsupported;
}

int aux_finalize(const float* partials, int nblocks, int E, long long T, const int32_t* tpe,
                 const float* lb_coef, int l_dtype, float* losses, void* f_i, int f_dtype,
                 float* p_i, void* z_out, cudaStream_t st) {
  if (E <= 0 || E > 256 || T <= 0 || nblocks <= 0) return kStatusBadArg;
  if (l_dtype == 0) return finalize_tf<__nv_bfloat16>(partials, nblocks, E, T, tpe, lb_coef, losses, f_i, f_dtype, p_i, z_out, st);
  if (l_dtype == 1) return finalize_tf<__half>(partials, nblocks, E, T, tpe, lb_coef, losses, f_i, f_dtype, p_i, z_out, st);
  if (l_dtype == 2) return finalize_tf<float>(partials, nblocks, E, T, tpe, lb_coef, losses, f_i, f_dtype, p_i, z_out, st);
  return kStatusUnsupported;
}

}  // namespace moe
