// Token permutation kernels (HBM-bound): padded gather, weighted padded
// gather, weighted top-k combine, relu^2 derivative, and the small index
// kernels that convert between the reference's sorted-order metadata and the
// padded-row maps the other kernels consume.
//
// Semantics follow triton_moe/kernels/gather.py:13-60,123-174 and
// triton_moe/kernels/scatter.py:13-69,104-133: padding rows are zero, a
// weighted row is round(x * w) in the storage dtype, and the combine sums the
// rounded per-expert products of a token in fp32 and rounds once.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "moe_internal.h"

namespace moe {
namespace {

template <typename T>
struct V8;  // 8 elements <-> uint4
template <>
struct V8<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const uint4& u, float (&f)[8]) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  static __device__ __forceinline__ uint4 store(const float (&f)[8]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    return u;
  }
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float rnd(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
  }
};
template <>
struct V8<__half> {
  static __device__ __forceinline__ void load(const uint4& u, float (&f)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __half22float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  static __device__ __forceinline__ uint4 store(const float (&f)[8]) {
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    return u;
  }
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float rnd(float v) { return __half2float(__float2half_rn(v)); }
};
// fp32 storage (used by the fp32 module path: plain copies, no rounding)
template <>
struct V8<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
  static __device__ __forceinline__ float rnd(float v) { return v; }
};

constexpr int kThreadsPerBlock = 256;

// The permutation kernels are launched with programmatic dependent launch:
// they wait for the previous grid before touching memory, and each block lets
// the next grid start launching once it has finished its own work (the next
// grid still waits for this one to complete before it touches memory).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_done() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

constexpr int kVecPerLane = 4;  // 16-byte vectors in flight per lane per batch

// out[r, :] = src row map[r] / div of x (times w[map[r]] when w != null);
// rows whose map entry is negative are zero.  Rows at or beyond *rows_dev
// (when given) are not touched.  A warp copies R consecutive rows at a time:
// lanes fetch the R map entries (and weights) together, then every lane
// issues all of its 16-byte loads for the R rows before the first store, so
// one memory round trip moves R rows.
template <typename T, bool VEC, int R>
__global__ void __launch_bounds__(kThreadsPerBlock)
    gather_rows_kernel(const T* __restrict__ x, long long ldx, int H,
                       const int32_t* __restrict__ map, int div, long long rows,
                       const int32_t* __restrict__ rows_dev, const T* __restrict__ w,
                       T* __restrict__ out, long long ldo) {
  pdl_wait();
  long long nrows = rows;
  if (rows_dev != nullptr) nrows = min(nrows, static_cast<long long>(*rows_dev));
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const long long wid = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  for (long long r0 = wid * R; r0 < nrows; r0 += warps * R) {
    // lane i < R: map entry and weight of row r0 + i
    int my_a = -1;
    float my_w = 1.f;
    if (lane < R && r0 + lane < nrows) {
      my_a = __ldg(map + r0 + lane);
      if (w != nullptr && my_a >= 0) my_w = V8<T>::to_f(w[my_a]);
    }
    int a[R];
    float sc[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      a[i] = __shfl_sync(0xffffffffu, my_a, i);
      sc[i] = __shfl_sync(0xffffffffu, my_w, i);
    }
    if constexpr (VEC) {
      for (int c0 = 0; c0 < H; c0 += 32 * 8 * kVecPerLane) {
        uint4 u[R][kVecPerLane];
#pragma unroll
        for (int i = 0; i < R; ++i)
#pragma unroll
          for (int j = 0; j < kVecPerLane; ++j) {
            const int c = c0 + (j * 32 + lane) * 8;
            u[i][j] = make_uint4(0, 0, 0, 0);
            if (a[i] >= 0 && c < H)
              u[i][j] = __ldg(reinterpret_cast<const uint4*>(
                  x + static_cast<long long>(a[i] / div) * ldx + c));
          }
#pragma unroll
        for (int i = 0; i < R; ++i) {
          if (r0 + i >= nrows) break;
          T* orow = out + (r0 + i) * ldo;
#pragma unroll
          for (int j = 0; j < kVecPerLane; ++j) {
            const int c = c0 + (j * 32 + lane) * 8;
            if (c >= H) break;
            if (w != nullptr && a[i] >= 0) {
              float f[8];
              V8<T>::load(u[i][j], f);
#pragma unroll
              for (int q = 0; q < 8; ++q) f[q] *= sc[i];
              u[i][j] = V8<T>::store(f);
            }
            *reinterpret_cast<uint4*>(orow + c) = u[i][j];
          }
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < R; ++i) {
        if (r0 + i >= nrows) break;
        T* orow = out + (r0 + i) * ldo;
        for (int c = lane; c < H; c += 32) {
          if (a[i] < 0) {
            orow[c] = V8<T>::from_f(0.f);
          } else {
            const T v = x[static_cast<long long>(a[i] / div) * ldx + c];
            orow[c] = w ? V8<T>::from_f(V8<T>::to_f(v) * sc[i]) : v;
          }
        }
      }
    }
  }
  pdl_done();
}

// out[t, :] = sum_j round(y[row(t,j), :] * w[t*k+j])  (fp32 sum, one rounding).
// A warp combines R tokens at a time: lanes fetch the R * kMaxK row indices
// and weights together, then all source-row vectors are loaded before any is
// used; NV 16-byte vectors per lane and source row cover 256*NV columns per
// pass (one pass for the usual hidden sizes).  Top-k beyond kMaxK runs in
// further batches of kMaxK.
template <typename T, bool VEC, int kMaxK, int R, int NV>
__global__ void __launch_bounds__(kThreadsPerBlock)
    combine_kernel(const T* __restrict__ y, long long ldy, int H,
                   const int32_t* __restrict__ asg_row, long long T_tokens, int k,
                   const T* __restrict__ w, T* __restrict__ out, long long ldo) {
  static_assert(R * kMaxK <= 32, "one lane per (token, source row)");
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const long long wid = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  for (long long t0 = wid * R; t0 < T_tokens; t0 += warps * R) {
    if constexpr (VEC) {
      for (int c0 = 0; c0 < H; c0 += 32 * 8 * NV) {
        float acc[R][NV][8];
#pragma unroll
        for (int i = 0; i < R; ++i)
#pragma unroll
          for (int v = 0; v < NV; ++v)
#pragma unroll
            for (int q = 0; q < 8; ++q) acc[i][v][q] = 0.f;
        for (int j0 = 0; j0 < k; j0 += kMaxK) {
          const int kk = min(kMaxK, k - j0);
          // lane l < R * kMaxK: source row and weight of (token l / kMaxK, j0 + l % kMaxK)
          int my_row = -1;
          float my_sc = 1.f;
          {
            const int ti = lane / kMaxK, jj = lane % kMaxK;
            if (lane < R * kMaxK && jj < kk && t0 + ti < T_tokens) {
              const long long ai = (t0 + ti) * k + j0 + jj;
              my_row = __ldg(asg_row + ai);
              if (w != nullptr) my_sc = V8<T>::to_f(w[ai]);
            }
          }
          int rows[R][kMaxK];
          float sc[R][kMaxK];
#pragma unroll
          for (int i = 0; i < R; ++i)
#pragma unroll
            for (int j = 0; j < kMaxK; ++j) {
              rows[i][j] = __shfl_sync(0xffffffffu, my_row, i * kMaxK + j);
              sc[i][j] = __shfl_sync(0xffffffffu, my_sc, i * kMaxK + j);
            }
          uint4 u[R][kMaxK][NV];
#pragma unroll
          for (int i = 0; i < R; ++i)
#pragma unroll
            for (int j = 0; j < kMaxK; ++j)
#pragma unroll
              for (int v = 0; v < NV; ++v) {
                const int c = c0 + (v * 32 + lane) * 8;
                if (rows[i][j] >= 0 && c < H)
                  u[i][j][v] = __ldg(reinterpret_cast<const uint4*>(y + rows[i][j] * ldy + c));
              }
#pragma unroll
          for (int i = 0; i < R; ++i)
#pragma unroll
            for (int j = 0; j < kMaxK; ++j) {
              if (rows[i][j] < 0) continue;
#pragma unroll
              for (int v = 0; v < NV; ++v) {
                if (c0 + (v * 32 + lane) * 8 >= H) continue;
                float f[8];
                V8<T>::load(u[i][j][v], f);
                if (w != nullptr) {
#pragma unroll
                  for (int q = 0; q < 8; ++q) acc[i][v][q] += V8<T>::rnd(f[q] * sc[i][j]);
                } else {
#pragma unroll
                  for (int q = 0; q < 8; ++q) acc[i][v][q] += f[q];
                }
              }
            }
        }
#pragma unroll
        for (int i = 0; i < R; ++i) {
          if (t0 + i >= T_tokens) break;
          T* orow = out + (t0 + i) * ldo;
#pragma unroll
          for (int v = 0; v < NV; ++v) {
            const int c = c0 + (v * 32 + lane) * 8;
            if (c < H) *reinterpret_cast<uint4*>(orow + c) = V8<T>::store(acc[i][v]);
          }
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const long long t = t0 + i;
        if (t >= T_tokens) break;
        T* orow = out + t * ldo;
        for (int c = lane; c < H; c += 32) {
          float acc = 0.f;
          for (int j = 0; j < k; ++j) {
            const int row = __ldg(asg_row + t * k + j);
            if (row < 0) continue;
            const float v = V8<T>::to_f(y[row * ldy + c]);
            acc += (w != nullptr) ? V8<T>::rnd(v * V8<T>::to_f(w[t * k + j])) : v;
          }
          orow[c] = V8<T>::from_f(acc);
        }
      }
    }
  }
  pdl_done();
}

// grad_act = pre > 0 ? round(g * 2 * pre) : 0, elementwise over [rows, cols].
template <typename T>
__global__ void relu2_grad_kernel(const T* __restrict__ g, const T* __restrict__ pre,
                                  long long rows, long long cols, long long ld,
                                  T* __restrict__ out) {
  const long long n = rows * cols;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / cols, c = i % cols;
    const float p = V8<T>::to_f(pre[r * ld + c]);
    const float gv = V8<T>::to_f(g[r * ld + c]);
    out[r * ld + c] = V8<T>::from_f(p > 0.f ? gv * 2.0f * p : 0.f);
  }
}

// SwiGLU backward, elementwise over [rows, w_e] per expert: from the output
// gradient g and the saved gate / up values,
//   s = sigmoid(gate), dgate = g * up * s * (1 + gate * (1 - s)), dup = g * gate * s,
// written (rounded) into grad_act[r, 0:w_e) and [w_e, 2 w_e) — the gate/up column
// layout of w1 — so the dX / dW GEMMs run over width 2 w_e.  One warp per row;
// the row's expert comes from a binary search over the token offsets.
template <typename T>
__global__ void swiglu_grad_kernel(const T* __restrict__ g, const T* __restrict__ gate,
                                   const T* __restrict__ up, long long rows, long long ld,
                                   const int32_t* __restrict__ tok_off,
                                   const int32_t* __restrict__ w_off, int E,
                                   T* __restrict__ out, long long ld_out) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const long long end = min(rows, static_cast<long long>(tok_off[E]));
  for (long long r = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       r < end; r += warps) {
    int lo = 0, hi = E - 1;  // last expert whose first row is <= r
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tok_off[mid] <= r) lo = mid;
      else hi = mid - 1;
    }
    const int w = (w_off[lo + 1] - w_off[lo]) / 2;
    for (int c = lane; c < w; c += 32) {
      const float gv = V8<T>::to_f(g[r * ld + c]);
      const float a = V8<T>::to_f(gate[r * ld + c]);
      const float u = V8<T>::to_f(up[r * ld + c]);
      const float sg = 1.0f / (1.0f + expf(-a));
      out[r * ld_out + c] = V8<T>::from_f(gv * u * sg * (1.0f + a * (1.0f - sg)));
      out[r * ld_out + w + c] = V8<T>::from_f(gv * a * sg);
    }
  }
  pdl_done();
}

// Sorted-order metadata -> padded row maps (row_asg pre-filled with -1).
__global__ void build_row_map_kernel(const int32_t* __restrict__ indices,
                                     const int32_t* __restrict__ bin_ids,
                                     const int32_t* __restrict__ bins,
                                     const int32_t* __restrict__ padded_bins, long long n_kept,
                                     long long p_rows, int32_t* __restrict__ row_asg,
                                     int32_t* __restrict__ asg_row, int* status) {
  for (long long p = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; p < n_kept;
       p += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int e = bin_ids[p];
    const long long bstart = e > 0 ? bins[e - 1] : 0;
    const long long pstart = e > 0 ? padded_bins[e - 1] : 0;
    const long long row = pstart + (p - bstart);
    const int a = indices[p];
    if (row < 0 || row >= p_rows) {
      if (status) atomicExch(status, kStatusCapacity);
      continue;
    }
    if (row_asg) row_asg[row] = a;
    if (asg_row) asg_row[a] = static_cast<int32_t>(row);
  }
}

// precompute_gather_map's format: padded row -> source token, padding rows 0.
__global__ void gather_map_kernel(const int32_t* __restrict__ row_asg, long long rows, int k,
                                  int32_t* __restrict__ gmap) {
  for (long long r = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; r < rows;
       r += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int a = row_asg[r];
    gmap[r] = a >= 0 ? a / k : 0;
  }
}

int grid_for(long long work_items, int per_block) {
  long long b = (work_items + per_block - 1) / per_block;
  const long long cap = static_cast<long long>(num_sms()) * 32;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return static_cast<int>(b);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename Kern, typename... Args>
int launch_pdl(Kern kern, int grid, cudaStream_t st, Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreadsPerBlock);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, args...) != cudaSuccess) return kStatusCuda;
  return cudaPeekAtLastError() == cudaSuccess ? kStatusOk : kStatusCuda;
}

template <typename T>
int gather_t(const void* x, long long ldx, int H, const int32_t* map, int div, long long rows,
             const int32_t* rows_dev, const void* w, void* out, long long ldo, cudaStream_t st) {
  if (rows <= 0 || H <= 0) return kStatusOk;
  const bool vec = H % 8 == 0 && ldx % 8 == 0 && ldo % 8 == 0 && aligned16(x) && aligned16(out);
  const T* xp = static_cast<const T*>(x);
  const T* wp = static_cast<const T*>(w);
  T* op = static_cast<T*>(out);
  constexpr int R = 1;  // rows per warp batch (more rows per warp measured slower)
  const int grid = grid_for((rows + R - 1) / R, kThreadsPerBlock / 32);
  if constexpr (sizeof(T) == 2) {
    if (vec)
      return launch_pdl(gather_rows_kernel<T, true, R>, grid, st, xp, ldx, H, map, div, rows,
                        rows_dev, wp, op, ldo);
  }
  return launch_pdl(gather_rows_kernel<T, false, R>, grid, st, xp, ldx, H, map, div, rows,
                    rows_dev, wp, op, ldo);
}

template <typename T>
int combine_t(const void* y, long long ldy, int H, const int32_t* asg_row, long long T_tokens,
              int k, const void* w, void* out, long long ldo, cudaStream_t st) {
  if (T_tokens <= 0 || H <= 0) return kStatusOk;
  const bool vec = H % 8 == 0 && ldy % 8 == 0 && ldo % 8 == 0 && aligned16(y) && aligned16(out);
  const T* yp = static_cast<const T*>(y);
  const T* wp = static_cast<const T*>(w);
  T* op = static_cast<T*>(out);
  // R tokens per warp batch and NV vectors per lane and source row: at most
  // 4 * 256 columns per pass for top-k <= 2, 2 * 256 beyond (register budget).
  // One token per warp measured faster than two at top-2 (more warps in flight).
  const int nv = (H + 255) / 256;
#define MOE_COMBINE_NV(KM, R, NV)                                                              \
  do {                                                                                         \
    const int grid = grid_for((T_tokens + (R) - 1) / (R), kThreadsPerBlock / 32);              \
    if constexpr (sizeof(T) == 2) {                                                            \
      if (vec)                                                                                 \
        return launch_pdl(combine_kernel<T, true, KM, R, NV>, grid, st, yp, ldy, H, asg_row,   \
                          T_tokens, k, wp, op, ldo);                                           \
    }                                                                                          \
    return launch_pdl(combine_kernel<T, false, KM, R, 1>, grid, st, yp, ldy, H, asg_row,       \
                      T_tokens, k, wp, op, ldo);                                               \
  } while (0)
#define MOE_COMBINE(KM, R)                \
  do {                                    \
    if (nv <= 1) MOE_COMBINE_NV(KM, R, 1); \
    if (nv <= 2) MOE_COMBINE_NV(KM, R, 2); \
    if (nv <= 3) MOE_COMBINE_NV(KM, R, 3); \
    MOE_COMBINE_NV(KM, R, 4);             \
  } while (0)
  if (k <= 1) MOE_COMBINE(1, 2);
  if (k <= 2) MOE_COMBINE(2, 1);
  if (k <= 4) MOE_COMBINE_NV(4, 1, 2);
  MOE_COMBINE_NV(8, 1, 2);
#undef MOE_COMBINE
#undef MOE_COMBINE_NV
}


}  // namespace

int swiglu_grad(const void* g, const void* gate, const void* up, long long rows, long long ld,
                const int32_t* tok_off, const int32_t* w_off, int E, void* out, long long ld_out,
                int dtype, cudaStream_t st) {
  if (rows <= 0) return kStatusOk;
  const int grid = grid_for(rows, kThreadsPerBlock / 32);
#define MOE_SWIGLU(T)                                                                        \
  return launch_pdl(swiglu_grad_kernel<T>, grid, st, static_cast<const T*>(g),               \
                    static_cast<const T*>(gate), static_cast<const T*>(up), rows, ld, tok_off, \
                    w_off, E, static_cast<T*>(out), ld_out)
  if (dtype == 0) MOE_SWIGLU(__nv_bfloat16);
  if (dtype == 1) MOE_SWIGLU(__half);
  if (dtype == 2) MOE_SWIGLU(float);
#undef MOE_SWIGLU
  return kStatusUnsupported;
}

// dtype: 0 bf16, 1 fp16, 2 fp32
int gather_rows(const void* x, long long ldx, int H, const int32_t* map, int div,
                long long rows, const int32_t* rows_dev, const void* w, void* out, long long ldo,
                int dtype, cudaStream_t st) {
  if (dtype == 0) return gather_t<__nv_bfloat16>(x, ldx, H, map, div, rows, rows_dev, w, out, ldo, st);
  if (dtype == 1) return gather_t<__half>(x, ldx, H, map, div, rows, rows_dev, w, out, ldo, st);
  if (dtype == 2) return gather_t<float>(x, ldx, H, map, div, rows, rows_dev, w, out, ldo, st);
  return kStatusUnsupported;
}

int combine_rows(const void* y, long long ldy, int H, const int32_t* asg_row, long long T_tokens,
                 int k, const void* w, void* out, long long ldo, int dtype, cudaStream_t st) {
  if (dtype == 0) return combine_t<__nv_bfloat16>(y, ldy, H, asg_row, T_tokens, k, w, out, ldo, st);
  if (dtype == 1) return combine_t<__half>(y, ldy, H, asg_row, T_tokens, k, w, out, ldo, st);
  if (dtype == 2) return combine_t<float>(y, ldy, H, asg_row, T_tokens, k, w, out, ldo, st);
  return kStatusUnsupported;
}

int relu2_grad(const void* g, const void* pre, long long rows, long long cols, long long ld,
               void* out, int dtype, cudaStream_t st) {
  if (rows <= 0 || cols <= 0) return kStatusOk;
  const int grid = grid_for(rows * cols, 256);
  if (dtype == 0)
    relu2_grad_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(g), static_cast<const __nv_bfloat16*>(pre), rows, cols,
        ld, static_cast<__nv_bfloat16*>(out));
  else if (dtype == 1)
    relu2_grad_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(g),
                                                    static_cast<const __half*>(pre), rows, cols,
                                                    ld, static_cast<__half*>(out));
  else if (dtype == 2)
    relu2_grad_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(g),
                                                   static_cast<const float*>(pre), rows, cols, ld,
                                                   static_cast<float*>(out));
  else
    return kStatusUnsupported;
  return cudaPeekAtLastError() == cudaSuccess ? kStatusOk : kStatusCuda;
}

int build_row_map(const int32_t* indices, const int32_t* bin_ids, const int32_t* bins,
                  const int32_t* padded_bins, long long n_kept, long long p_rows,
                  int32_t* row_asg, long long n_asg, int32_t* asg_row, int* status,
                  cudaStream_t st) {
  if (row_asg && p_rows > 0) cudaMemsetAsync(row_asg, 0xFF, p_rows * 4, st);
  if (asg_row && n_asg > 0) cudaMemsetAsync(asg_row, 0xFF, n_asg * 4, st);
  if (n_kept > 0)
    build_row_map_kernel<<<grid_for(n_kept, 256), 256, 0, st>>>(
        indices, bin_ids, bins, padded_bins, n_kept, p_rows, row_asg, asg_row, status);
  return cudaPeekAtLastError() == cudaSuccess ? kStatusOk : kStatusCuda;
}

int gather_map_from_rows(const int32_t* row_asg, long long rows, int k, int32_t* gmap,
                         cudaStream_t st) {
  if (rows <= 0) return kStatusOk;
  gather_map_kernel<<<grid_for(rows, 256), 256, 0, st>>>(row_asg, rows, k, gmap);
  return cudaPeekAtLastError() == cudaSuccess ? kStatusOk : kStatusCuda;
}

}  // namespace moe
