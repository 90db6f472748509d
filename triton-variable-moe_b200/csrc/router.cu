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
