// Expert parallelism: the token exchange between the ranks that share one
// layer's experts, over NVLink peer memory.
//
// The reference runs every expert on one GPU (triton_moe/moe.py:185-249).
// Sharded, each rank routes its own tokens; an expert's rows travel to the
// rank that owns it and its outputs travel back:
//   dispatch : a push kernel reads each of this rank's token rows (the
//              gather, fused) and stores it straight into the owner's padded,
//              expert-contiguous layout (the rows the grouped GEMMs read) in
//              the owner's memory, mapped here through CUDA IPC;
//   combine  : a pull kernel forms each token's weighted top-k sum from the
//              owners' output rows, read over NVLink (the scatter, fused).
// No re-ordering pass runs on either side.  Ranks order their accesses to
// each other's buffers with a barrier (a one-word NCCL all-reduce on the
// stream) before a buffer is written and before it is read.  Tokens may be
// split into chunks so that the GEMMs of one chunk overlap the transfers of
// its neighbours.
//
// Layout of the per-(source, chunk, expert) row counts every rank holds
// after the count exchange: counts[s][c][e], int32, s < world, c < chunks,
// e < num_experts (global ids).  A rank's local experts are the ids it owns,
// in ascending order.
//
// NCCL is resolved at run time (dlopen/dlsym): the library has no link-time
// dependency on it, and inside a process that already loaded NCCL (e.g.
// PyTorch's) that copy is used.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <vector>

#include "moe_b200.h"

namespace {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // a copy already loaded
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (h == nullptr) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (h == nullptr) return;
    auto sym = [h](const char* n) { return dlsym(h, n); };
    api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(sym("ncclGetUniqueId"));
    api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(sym("ncclCommInitRank"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(sym("ncclCommDestroy"));
    api.AllGather = reinterpret_cast<decltype(api.AllGather)>(sym("ncclAllGather"));
    api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(sym("ncclAllReduce"));
    api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.AllGather &&
             api.AllReduce;
  });
  return api;
}

bool plan_args_ok(int world, int rank, int chunks, int num_experts, const int32_t* owner,
                  const int32_t* counts) {
  if (world < 1 || rank < 0 || rank >= world || chunks < 1 || num_experts < 1 || !owner ||
      !counts)
    return false;
  for (int e = 0; e < num_experts; ++e)
    if (owner[e] < 0 || owner[e] >= world) return false;
  return true;
}

// Global ids of the experts `rank` owns, ascending.
std::vector<int> local_experts(int rank, int num_experts, const int32_t* owner) {
  std::vector<int> v;
  for (int e = 0; e < num_experts; ++e)
    if (owner[e] == rank) v.push_back(e);
  return v;
}

inline int64_t cnt(const int32_t* counts, int chunks, int E, int s, int c, int e) {
  return counts[(static_cast<int64_t>(s) * chunks + c) * E + e];
}

// ---- device side -----------------------------------------------------------
// 16-byte vectors of N elements; weighted values are round(v * w) in the
// storage type, and the combine sums the rounded products of a token's rows
// in fp32 and rounds once (the rounding points of the single-GPU gather and
// combine kernels, triton_moe/kernels/gather.py:170-174, scatter.py:61-69).
template <typename T>
struct Vec;
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void unpack(const uint4& u, float* f) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  static __device__ __forceinline__ uint4 pack(const float* f) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    return u;
  }
  static __device__ __forceinline__ float rnd(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
  }
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
};
template <>
struct Vec<__half> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void unpack(const uint4& u, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __half22float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  static __device__ __forceinline__ uint4 pack(const float* f) {
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    return u;
  }
  static __device__ __forceinline__ float rnd(float v) { return __half2float(__float2half_rn(v)); }
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
};
template <>
struct Vec<float> {
  static constexpr int N = 4;
  static __device__ __forceinline__ void unpack(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  }
  static __device__ __forceinline__ uint4 pack(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  }
  static __device__ __forceinline__ float rnd(float v) { return v; }
  static __device__ __forceinline__ float to_f(float v) { return v; }
};

constexpr int kEpThreads = 256;
constexpr int kPushVec = 4;  // 16-byte vectors per lane loaded before they are stored

template <typename T>
__device__ __forceinline__ T* peer_base(T* const* peers, int r) {
  return reinterpret_cast<T*>(__ldg(reinterpret_cast<const unsigned long long*>(peers + r)));
}

// Dispatch push: row i of this rank's expert-sorted rows (routing with block
// size 1: assignment r2a[i] = t * k + j, expert bin_ids[i]) is token t of x,
// times w[r2a[i]] when w is given; it goes to row i + delta[e] of the owner
// e's layout, in the owner's memory (peers[owner[e]]).  One warp per row.
template <typename T>
__global__ void __launch_bounds__(kEpThreads)
    ep_push_kernel(const T* __restrict__ x, long long ldx, int H, const int32_t* __restrict__ r2a,
                   int k, const T* __restrict__ w, const int32_t* __restrict__ bin_ids,
                   long long rows, const int32_t* __restrict__ owner,
                   const long long* __restrict__ delta, T* const* __restrict__ peers,
                   long long ldp) {
  constexpr int N = Vec<T>::N;
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long i = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       i < rows; i += warps) {
    const int a = __ldg(r2a + i);
    const int e = __ldg(bin_ids + i);
    const T* src = x + static_cast<long long>(a / k) * ldx;
    T* dst = peer_base(peers, __ldg(owner + e)) + (i + __ldg(delta + e)) * ldp;
    const float sc = w != nullptr ? Vec<T>::to_f(w[a]) : 1.f;
    for (int c0 = 0; c0 < H; c0 += 32 * N * kPushVec) {
      uint4 u[kPushVec];
#pragma unroll
      for (int j = 0; j < kPushVec; ++j) {
        const int c = c0 + (j * 32 + lane) * N;
        if (c < H) u[j] = __ldg(reinterpret_cast<const uint4*>(src + c));
      }
#pragma unroll
      for (int j = 0; j < kPushVec; ++j) {
        const int c = c0 + (j * 32 + lane) * N;
        if (c >= H) break;
        if (w != nullptr) {
          float f[N];
          Vec<T>::unpack(u[j], f);
#pragma unroll
          for (int q = 0; q < N; ++q) f[q] *= sc;
          u[j] = Vec<T>::pack(f);
        }
        *reinterpret_cast<uint4*>(dst + c) = u[j];
      }
    }
  }
  // the stores to peer memory are performed before the barrier that follows
  __threadfence_system();
}

// Combine pull: out[t] = sum_j round(Y[row(t, j)] * w[t*k + j]) (unit weights
// when w is null), fp32 sum rounded once, where assignment a = t*k + j sits at
// row asg_row[a] of this rank's expert-sorted rows, its expert is e =
// bin_ids[asg_row[a]], and its output row is asg_row[a] + delta[e] of the
// owner's layout, read from the owner's memory (peers[owner[e]]).  One warp
// per token; every source row's vectors of a column pass are loaded before
// any is summed.
constexpr int kPullK = 8;   // source rows loaded together
constexpr int kPullVec = 2;  // 16-byte vectors per lane and source row per pass
template <typename T>
__global__ void __launch_bounds__(kEpThreads, 2)
    ep_pull_combine_kernel(T* const* __restrict__ peers, long long ldp,
                           const int32_t* __restrict__ owner, const long long* __restrict__ delta,
                           const int32_t* __restrict__ bin_ids, const int32_t* __restrict__ asg_row,
                           long long tokens, int k, const T* __restrict__ w, int H,
                           T* __restrict__ out, long long ldo) {
  constexpr int N = Vec<T>::N;
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long t = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       t < tokens; t += warps) {
    for (int c0 = 0; c0 < H; c0 += 32 * N * kPullVec) {
      float acc[kPullVec][N];
#pragma unroll
      for (int v = 0; v < kPullVec; ++v)
#pragma unroll
        for (int q = 0; q < N; ++q) acc[v][q] = 0.f;
      for (int j0 = 0; j0 < k; j0 += kPullK) {
        const int kk = min(kPullK, k - j0);
        // lane j < kk: the source row and weight of assignment j0 + j
        const T* my_src = nullptr;
        float my_sc = 1.f;
        if (lane < kk) {
          const long long a = t * k + j0 + lane;
          const int r = __ldg(asg_row + a);
          if (r >= 0) {
            const int e = __ldg(bin_ids + r);
            my_src = peer_base(peers, __ldg(owner + e)) + (r + __ldg(delta + e)) * ldp;
          }
          if (w != nullptr) my_sc = Vec<T>::to_f(w[a]);
        }
        const T* src[kPullK];
        float sc[kPullK];
#pragma unroll
        for (int j = 0; j < kPullK; ++j) {
          src[j] = reinterpret_cast<const T*>(
              __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(my_src), j));
          sc[j] = __shfl_sync(0xffffffffu, my_sc, j);
        }
        uint4 u[kPullK][kPullVec];
#pragma unroll
        for (int j = 0; j < kPullK; ++j)
#pragma unroll
          for (int v = 0; v < kPullVec; ++v) {
            const int c = c0 + (v * 32 + lane) * N;
            if (src[j] != nullptr && c < H)
              u[j][v] = *reinterpret_cast<const uint4*>(src[j] + c);
          }
#pragma unroll
        for (int j = 0; j < kPullK; ++j) {
          if (src[j] == nullptr) continue;
#pragma unroll
          for (int v = 0; v < kPullVec; ++v) {
            if (c0 + (v * 32 + lane) * N >= H) continue;
            float f[N];
            Vec<T>::unpack(u[j][v], f);
            if (w != nullptr) {
#pragma unroll
              for (int q = 0; q < N; ++q) acc[v][q] += Vec<T>::rnd(f[q] * sc[j]);
            } else {
#pragma unroll
              for (int q = 0; q < N; ++q) acc[v][q] += f[q];
            }
          }
        }
      }
#pragma unroll
      for (int v = 0; v < kPullVec; ++v) {
        const int c = c0 + (v * 32 + lane) * N;
        if (c < H) *reinterpret_cast<uint4*>(out + t * ldo + c) = Vec<T>::pack(acc[v]);
      }
    }
  }
}

int launch_grid(long long work) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long per = kEpThreads / 32;
  const long long need = (work + per - 1) / per;
  return static_cast<int>(need < 4LL * sms ? (need > 0 ? need : 1) : 4LL * sms);
}

bool vec_ok(int dtype, int64_t hidden, int64_t ld_a, int64_t ld_b, const void* p) {
  const int es = dtype == MOE_DTYPE_F32 ? 4 : 2;
  return (hidden * es) % 16 == 0 && (ld_a * es) % 16 == 0 && (ld_b * es) % 16 == 0 &&
         (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

}  // namespace

extern "C" {

int moe_ep_unique_id(void* id) {
  const NcclApi& api = nccl();
  if (!api.ok) return MOE_ERR_COMM;
  if (!id) return MOE_ERR_BAD_ARG;
  ncclUniqueId u;
  if (api.GetUniqueId(&u) != ncclSuccess) return MOE_ERR_COMM;
  std::memcpy(id, &u, sizeof(u));
  return MOE_OK;
}

int moe_ep_comm_init(void** comm, const void* id, int world, int rank) {
  const NcclApi& api = nccl();
  if (!api.ok) return MOE_ERR_COMM;
  if (!comm || !id || world < 1 || rank < 0 || rank >= world) return MOE_ERR_BAD_ARG;
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  ncclComm_t c = nullptr;
  if (api.CommInitRank(&c, world, u, rank) != ncclSuccess) return MOE_ERR_COMM;
  *comm = c;
  return MOE_OK;
}

int moe_ep_comm_destroy(void* comm) {
  const NcclApi& api = nccl();
  if (!api.ok) return MOE_ERR_COMM;
  if (!comm) return MOE_ERR_BAD_ARG;
  return api.CommDestroy(static_cast<ncclComm_t>(comm)) == ncclSuccess ? MOE_OK : MOE_ERR_COMM;
}

int moe_ep_gather_counts(void* comm, const int32_t* mine, int32_t* all, int64_t n,
                         void* stream) {
  const NcclApi& api = nccl();
  if (!api.ok) return MOE_ERR_COMM;
  if (!comm || !mine || !all || n < 0) return MOE_ERR_BAD_ARG;
  if (n == 0) return MOE_OK;
  return api.AllGather(mine, all, static_cast<size_t>(n), ncclInt32,
                       static_cast<ncclComm_t>(comm),
                       static_cast<cudaStream_t>(stream)) == ncclSuccess
             ? MOE_OK
             : MOE_ERR_COMM;
}

int moe_ep_barrier(void* comm, int32_t* word, void* stream) {
  const NcclApi& api = nccl();
  if (!api.ok) return MOE_ERR_COMM;
  if (!comm || !word) return MOE_ERR_BAD_ARG;
  return api.AllReduce(word, word, 1, ncclInt32, ncclMax, static_cast<ncclComm_t>(comm),
                       static_cast<cudaStream_t>(stream)) == ncclSuccess
             ? MOE_OK
             : MOE_ERR_COMM;
}

int moe_ep_buffer_create(int64_t bytes, void** ptr, void* ipc_handle) {
  if (bytes <= 0 || !ptr || !ipc_handle) return MOE_ERR_BAD_ARG;
  void* p = nullptr;
  if (cudaMalloc(&p, static_cast<size_t>(bytes)) != cudaSuccess) return MOE_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return MOE_ERR_CUDA;
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return MOE_OK;
}

int moe_ep_buffer_free(void* ptr) {
  if (!ptr) return MOE_ERR_BAD_ARG;
  return cudaFree(ptr) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

int moe_ep_buffer_open(const void* ipc_handle, void** ptr) {
  if (!ipc_handle || !ptr) return MOE_ERR_BAD_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess
             ? MOE_OK
             : MOE_ERR_CUDA;
}

int moe_ep_buffer_close(void* ptr) {
  if (!ptr) return MOE_ERR_BAD_ARG;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

int moe_ep_plan(int world, int rank, int chunks, int num_experts, int block_size,
                const int32_t* owner, const int32_t* counts, int64_t* src_off,
                int32_t* tok_off, int32_t* chunk_off, int32_t* chunk_rows, int64_t* recv_off) {
  if (!plan_args_ok(world, rank, chunks, num_experts, owner, counts) || block_size < 1 ||
      !src_off || !tok_off || !chunk_off || !chunk_rows || !recv_off)
    return MOE_ERR_BAD_ARG;
  const int E = num_experts;
  for (int64_t i = 0; i < static_cast<int64_t>(world) * chunks * E; ++i)
    if (counts[i] < 0) return MOE_ERR_BAD_ARG;
  const std::vector<int> mine = local_experts(rank, E, owner);
  const int el = static_cast<int>(mine.size());
  // this rank's rows of each chunk, expert-sorted (block size 1)
  for (int c = 0; c < chunks; ++c) {
    int64_t run = 0;
    for (int e = 0; e < E; ++e) {
      src_off[static_cast<int64_t>(c) * E + e] = run;
      run += cnt(counts, chunks, E, rank, c, e);
    }
  }
  // the owner's layout: one region per local expert; in it one block per
  // chunk, each holding the sources' rows in rank order and rounded up to
  // the block size
  int64_t pos = 0;
  for (int li = 0; li < el; ++li) {
    tok_off[li] = static_cast<int32_t>(pos);
    for (int c = 0; c < chunks; ++c) {
      chunk_off[static_cast<int64_t>(c) * (el + 1) + li] = static_cast<int32_t>(pos);
      int64_t tot = 0;
      for (int s = 0; s < world; ++s) {
        recv_off[(static_cast<int64_t>(s) * chunks + c) * el + li] = pos + tot;
        tot += cnt(counts, chunks, E, s, c, mine[li]);
      }
      const int64_t padded = (tot + block_size - 1) / block_size * block_size;
      chunk_rows[static_cast<int64_t>(c) * el + li] = static_cast<int32_t>(padded);
      pos += padded;
      if (pos > INT32_MAX) return MOE_ERR_CAPACITY;
    }
  }
  tok_off[el] = static_cast<int32_t>(pos);
  for (int c = 0; c < chunks; ++c)
    chunk_off[static_cast<int64_t>(c) * (el + 1) + el] = static_cast<int32_t>(pos);
  return MOE_OK;
}

int moe_ep_dispatch(const void* x, int64_t ld_x, int64_t hidden, const int32_t* row_to_assignment,
                    int top_k, const void* weights, const int32_t* bin_ids, int64_t rows,
                    const int32_t* owner, const int64_t* delta, void* const* peers,
                    int64_t ld_peer, int dtype, void* stream) {
  if (rows < 0 || hidden <= 0 || top_k < 1 ||
      (rows > 0 && (!x || !row_to_assignment || !bin_ids || !owner || !delta || !peers)))
    return MOE_ERR_BAD_ARG;
  if (!vec_ok(dtype, hidden, ld_x, ld_peer, x)) return MOE_ERR_BAD_ARG;
  if (rows == 0) return MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = launch_grid(rows);
  const int H = static_cast<int>(hidden);
  const auto* d = reinterpret_cast<const long long*>(delta);
  if (dtype == MOE_DTYPE_BF16)
    ep_push_kernel<__nv_bfloat16><<<grid, kEpThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), ld_x, H, row_to_assignment, top_k,
        static_cast<const __nv_bfloat16*>(weights), bin_ids, rows, owner, d,
        reinterpret_cast<__nv_bfloat16* const*>(peers), ld_peer);
  else if (dtype == MOE_DTYPE_F16)
    ep_push_kernel<__half><<<grid, kEpThreads, 0, st>>>(
        static_cast<const __half*>(x), ld_x, H, row_to_assignment, top_k,
        static_cast<const __half*>(weights), bin_ids, rows, owner, d,
        reinterpret_cast<__half* const*>(peers), ld_peer);
  else if (dtype == MOE_DTYPE_F32)
    ep_push_kernel<float><<<grid, kEpThreads, 0, st>>>(
        static_cast<const float*>(x), ld_x, H, row_to_assignment, top_k,
        static_cast<const float*>(weights), bin_ids, rows, owner, d,
        reinterpret_cast<float* const*>(peers), ld_peer);
  else
    return MOE_ERR_UNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

int moe_ep_combine(void* const* peers, int64_t ld_peer, const int32_t* owner,
                   const int64_t* delta, const int32_t* bin_ids,
                   const int32_t* assignment_to_row, int64_t num_tokens, int top_k,
                   const void* weights, int64_t hidden, void* out, int64_t ld_out, int dtype,
                   void* stream) {
  if (num_tokens < 0 || hidden <= 0 || top_k < 1 ||
      (num_tokens > 0 && (!peers || !owner || !delta || !bin_ids || !assignment_to_row || !out)))
    return MOE_ERR_BAD_ARG;
  if (!vec_ok(dtype, hidden, ld_out, ld_peer, out)) return MOE_ERR_BAD_ARG;
  if (num_tokens == 0) return MOE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = launch_grid(num_tokens);
  const int H = static_cast<int>(hidden);
  const auto* d = reinterpret_cast<const long long*>(delta);
  if (dtype == MOE_DTYPE_BF16)
    ep_pull_combine_kernel<__nv_bfloat16><<<grid, kEpThreads, 0, st>>>(
        reinterpret_cast<__nv_bfloat16* const*>(peers), ld_peer, owner, d, bin_ids,
        assignment_to_row, num_tokens, top_k, static_cast<const __nv_bfloat16*>(weights), H,
        static_cast<__nv_bfloat16*>(out), ld_out);
  else if (dtype == MOE_DTYPE_F16)
    ep_pull_combine_kernel<__half><<<grid, kEpThreads, 0, st>>>(
        reinterpret_cast<__half* const*>(peers), ld_peer, owner, d, bin_ids, assignment_to_row,
        num_tokens, top_k, static_cast<const __half*>(weights), H, static_cast<__half*>(out),
        ld_out);
  else if (dtype == MOE_DTYPE_F32)
    ep_pull_combine_kernel<float><<<grid, kEpThreads, 0, st>>>(
        reinterpret_cast<float* const*>(peers), ld_peer, owner, d, bin_ids, assignment_to_row,
        num_tokens, top_k, static_cast<const float*>(weights), H, static_cast<float*>(out),
        ld_out);
  else
    return MOE_ERR_UNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

}  // extern "C"
