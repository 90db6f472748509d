// Routing: histogram, rounded bin offsets and a stable counting sort of the
// top-k expert assignments into expert-contiguous order.
//
// Restates triton_moe/kernels/fused_cumsum.py:84-171 (torch.sort(stable) +
// torch.bincount + _cumsum_kernel, with the "down"/"nearest" compaction of
// :154-169 done on device) and precompute_gather_map
// (triton_moe/kernels/grouped_gemm.py:104-149) without any host sync.
//
// Work is split into "units": contiguous runs of assignments, one warp each.
//   count        : per-unit per-expert histogram          -> ws[unit][E]
//   scan+scatter : every block derives its units' starting ranks, the expert
//                  totals, rounding and offsets from the histograms itself
//                  (block 0 also writes the per-expert outputs and padding-row
//                  markers), then each warp ranks its unit stably (match_any)
//                  and writes the sorted order and both row maps
// Problems of at most 6144 assignments run all phases in one CTA (its time grows
// with the assignments; past ~7000 the two multi-block launches are faster).
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "moe_internal.h"

namespace moe {
namespace {

constexpr int kMaxE = 256;
constexpr int kWarpsPerBlock = 8;
constexpr int kBatch = 8;  // warp-steps of ids loaded together per lane

struct RouteOut {
  int32_t* bin_ids;
  int32_t* indices;
  int32_t* tpe;
  int32_t* bins;
  int32_t* padded_bins;
  int32_t* tok_off;
  int32_t* ptpe;
  int32_t* row_asg;
  long long p_cap;
  int32_t* asg_row;
  int* status;
};

__device__ __forceinline__ int rounded_count(int n, int bs, int mode) {
  if (mode == 0) return ((n + bs - 1) / bs) * bs;
  if (mode == 1) return (n / bs) * bs;
  return ((n + bs / 2) / bs) * bs;
}

// ---- phase 1: per-unit histograms -------------------------------------------
template <typename S>
__global__ void route_count_kernel(const S* __restrict__ sel, long long A, int E, long long U,
                                   long long units, int32_t* __restrict__ ws, int* status) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ int hist[kWarpsPerBlock][kMaxE];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long unit = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + w;
  for (int e = lane; e < E; e += 32) hist[w][e] = 0;
  __syncwarp();
  if (unit < units) {
    const long long beg = unit * U, end = min(A, beg + U);
    // kBatch independent loads in flight per lane before the shared atomics
    for (long long i0 = beg + lane; i0 < end; i0 += 32LL * kBatch) {
      S v[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const long long i = i0 + 32LL * j;
        v[j] = i < end ? sel[i] : S(0);
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const long long i = i0 + 32LL * j;
        if (i < end) {
          const long long e = static_cast<long long>(v[j]);
          if (e < 0 || e >= E) {
            if (status) atomicExch(status, kStatusBadExpert);
          } else {
            atomicAdd(&hist[w][e], 1);
          }
        }
      }
    }
    __syncwarp();
    for (int e = lane; e < E; e += 32) ws[unit * E + e] = hist[w][e];
  }
}

// Block-wide exclusive scan of one int per thread (blockDim.x <= 1024).
__device__ int block_excl_scan(int v, int* total) {
  __shared__ int warp_sums[32];
  __shared__ int block_total;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) warp_sums[w] = incl;
  __syncthreads();
  if (w == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    int s = lane < nw ? warp_sums[lane] : 0;
    int si = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int t = __shfl_up_sync(0xffffffffu, si, o);
      if (lane >= o) si += t;
    }
    if (lane < nw) warp_sums[lane] = si - s;
    if (lane == nw - 1) block_total = si;
  }
  __syncthreads();
  const int res = warp_sums[w] + incl - v;
  const int tot = block_total;
  __syncthreads();
  if (total) *total = tot;
  return res;
}

// ---- phase 2: scan + stable scatter ------------------------------------------------
// Every block (8 warps = 8 units) computes what it needs from the per-unit
// histograms itself: each expert's total and the count of its assignments in
// units before the block (threads split the units of an expert between them),
// the expert-level rounding and cumulative sums, and its warps' starting
// ranks.  Block 0 also writes the per-expert outputs and marks padding rows.
// Then each warp ranks its unit's assignments stably (match_any) and scatters
// them.
template <typename S>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    route_scan_scatter_kernel(const S* __restrict__ sel, long long A, int E, int bs, int mode,
                              long long U, long long units, const int32_t* __restrict__ ws,
                              RouteOut o) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ int base[kWarpsPerBlock][kMaxE];
  __shared__ int s_tot[kMaxE], s_before[kMaxE];
  __shared__ int s_bstart[kMaxE], s_pstart[kMaxE], s_kept[kMaxE], s_padpre[kMaxE + 1];
  __shared__ int s_part[kWarpsPerBlock * 32], s_part2[kWarpsPerBlock * 32];
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int nthr = kWarpsPerBlock * 32;
  const long long u0 = static_cast<long long>(blockIdx.x) * kWarpsPerBlock;
  // (a) per-expert totals and counts before this block's first unit
  const int parts = max(1, nthr / E);
  const int groups = nthr / parts;
  for (int e0 = 0; e0 < E; e0 += groups) {
    const int g = tid / parts, part = tid % parts;
    const int e = e0 + g;
    int tot = 0, bef = 0;
    if (g < groups && e < E) {
#pragma unroll 4
      for (long long u = part; u < units; u += parts) {
        const int c = ws[u * E + e];
        tot += c;
        if (u < u0) bef += c;
      }
    }
    s_part[tid] = tot;
    s_part2[tid] = bef;
    __syncthreads();
    if (g < groups && e < E && part == 0) {
      int t2 = 0, b2 = 0;
      for (int q = 0; q < parts; ++q) {
        t2 += s_part[tid + q];
        b2 += s_part2[tid + q];
      }
      s_tot[e] = t2;
      s_before[e] = b2;
    }
    __syncthreads();
  }
  // (b) starting rank of each warp's unit per expert
  for (int e = tid; e < E; e += nthr) {
    int run = s_before[e];
    for (int ww = 0; ww < kWarpsPerBlock; ++ww) {
      base[ww][e] = run;
      if (u0 + ww < units) run += ws[(u0 + ww) * E + e];
    }
  }
  // (c) expert level: rounding and the cumulative sums (thread e holds expert e)
  int n = 0, r = 0, kept = 0, pads = 0;
  if (tid < E) {
    n = s_tot[tid];
    r = rounded_count(n, bs, mode);
    kept = min(n, r);
    pads = r - kept;
  }
  int tot_kept, tot_round, tot_pad;
  const int kept_ex = block_excl_scan(kept, &tot_kept);
  const int round_ex = block_excl_scan(r, &tot_round);
  const int pad_ex = block_excl_scan(pads, &tot_pad);
  if (tid < E) {
    s_kept[tid] = kept;
    s_pstart[tid] = round_ex;
    s_bstart[tid] = kept_ex;
    s_padpre[tid] = pad_ex;
    if (blockIdx.x == 0) {
      o.tpe[tid] = n;
      o.bins[tid] = kept_ex + kept;
      o.padded_bins[tid] = round_ex + r;
      o.tok_off[tid] = round_ex;
      o.ptpe[tid] = r;
      if (tid == E - 1) o.tok_off[E] = round_ex + r;
    }
  }
  __syncthreads();
  const bool write_rows = o.row_asg != nullptr && static_cast<long long>(tot_round) <= o.p_cap;
  if (blockIdx.x == 0) {
    if (o.row_asg != nullptr && !write_rows && tid == 0 && o.status)
      atomicExch(o.status, kStatusCapacity);
    if (write_rows) {
      for (int p = tid; p < tot_pad; p += nthr) {
        int lo = 0, hi = E - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (s_padpre[mid] <= p) lo = mid;
          else hi = mid - 1;
        }
        o.row_asg[s_pstart[lo] + s_kept[lo] + (p - s_padpre[lo])] = -1;
      }
    }
  }
  // (d) stable scatter of this warp's unit
  const long long unit = u0 + w;
  if (unit < units) {
    const long long beg = unit * U, end = min(A, beg + U);
    int ev[kBatch];
    for (long long i0 = beg; i0 < end; i0 += 32) {
      const long long i = i0 + lane;
      const bool valid = i < end;
      const int jb = static_cast<int>(((i0 - beg) >> 5) % kBatch);
      if (jb == 0) {
        // the next kBatch warp-steps' ids, all loads in flight together
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          const long long ij = i + 32LL * j;
          ev[j] = -1;
          if (ij < end) {
            const long long v = static_cast<long long>(sel[ij]);
            ev[j] = (v >= 0 && v < E) ? static_cast<int>(v) : -1;
          }
        }
      }
      int e = -1;
#pragma unroll
      for (int j = 0; j < kBatch; ++j)
        if (j == jb) e = ev[j];
      if (!valid) e = -1;
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      const int rank_in = __popc(peers & ((1u << lane) - 1u));
      if (e >= 0) {
        const int rank = base[w][e] + rank_in;
        if (rank < s_kept[e]) {
          const int pos = s_bstart[e] + rank;
          o.bin_ids[pos] = e;
          o.indices[pos] = static_cast<int32_t>(i);
          const int row = s_pstart[e] + rank;
          if (write_rows) o.row_asg[row] = static_cast<int32_t>(i);
          if (o.asg_row) o.asg_row[i] = row;
        } else if (o.asg_row) {
          o.asg_row[i] = -1;  // dropped by "down"/"nearest" rounding
        }
      } else if (valid && o.asg_row) {
        o.asg_row[i] = -1;
      }
      __syncwarp();
      if (e >= 0 && lane == 31 - __clz(peers)) base[w][e] += __popc(peers);
      __syncwarp();
    }
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- single-CTA path for small problems ------------------------------------------
// All three phases in one CTA of 32 warps (one launch instead of three): warp w
// owns the contiguous chunk [w*U, (w+1)*U) of assignments; its per-expert
// histogram row in shared memory becomes its running rank base.
constexpr int kSmallWarps = 32;
constexpr long long kSmallMaxA = 6144;

template <typename S>
__global__ void __launch_bounds__(kSmallWarps * 32, 1)
    route_small_kernel(const S* __restrict__ sel, long long A, int E, int bs, int mode,
                       RouteOut o) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ int hist[kSmallWarps][kMaxE];
  __shared__ int s_kept[kMaxE], s_pstart[kMaxE], s_bstart[kMaxE], s_padpre[kMaxE + 1];
  extern __shared__ int16_t s_sel[];  // [A] expert id of every assignment (-1: invalid)
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  for (int i = tid; i < kSmallWarps * kMaxE; i += blockDim.x) (&hist[0][0])[i] = 0;
  // one coalesced pass over the ids, eight independent loads in flight per thread
  for (long long i0 = 0; i0 < A; i0 += 8LL * blockDim.x) {
    S v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const long long i = i0 + j * blockDim.x + tid;
      v[j] = i < A ? sel[i] : S(0);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const long long i = i0 + j * blockDim.x + tid;
      if (i < A) {
        const long long e = static_cast<long long>(v[j]);
        const bool ok = e >= 0 && e < E;
        if (!ok && o.status) atomicExch(o.status, kStatusBadExpert);
        s_sel[i] = ok ? static_cast<int16_t>(e) : static_cast<int16_t>(-1);
      }
    }
  }
  __syncthreads();
  const long long U = ((A + kSmallWarps - 1) / kSmallWarps + 31) / 32 * 32;
  const long long beg = w * U, end = min(A, beg + U);
  for (long long i = beg + lane; i < end; i += 32) {
    const int e = s_sel[i];
    if (e >= 0) atomicAdd(&hist[w][e], 1);
  }
  __syncthreads();
  int n = 0;
  if (tid < E) {
    for (int ww = 0; ww < kSmallWarps; ++ww) {
      const int c = hist[ww][tid];
      hist[ww][tid] = n;
      n += c;
    }
  }
  int r = 0, kept = 0, pads = 0;
  if (tid < E) {
    r = rounded_count(n, bs, mode);
    kept = min(n, r);
    pads = r - kept;
  }
  int tot_kept, tot_round, tot_pad;
  const int kept_ex = block_excl_scan(kept, &tot_kept);
  const int round_ex = block_excl_scan(r, &tot_round);
  const int pad_ex = block_excl_scan(pads, &tot_pad);
  if (tid < E) {
    s_kept[tid] = kept;
    s_pstart[tid] = round_ex;
    s_bstart[tid] = kept_ex;
    s_padpre[tid] = pad_ex;
    o.tpe[tid] = n;
    o.bins[tid] = kept_ex + kept;
    o.padded_bins[tid] = round_ex + r;
    o.tok_off[tid] = round_ex;
    o.ptpe[tid] = r;
    if (tid == E - 1) o.tok_off[E] = round_ex + r;
  }
  __syncthreads();
  const bool write_rows = o.row_asg != nullptr && static_cast<long long>(tot_round) <= o.p_cap;
  if (o.row_asg != nullptr && !write_rows && tid == 0 && o.status)
    atomicExch(o.status, kStatusCapacity);
  if (write_rows) {
    for (int p = tid; p < tot_pad; p += blockDim.x) {
      int lo = 0, hi = E - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_padpre[mid] <= p) lo = mid;
        else hi = mid - 1;
      }
      o.row_asg[s_pstart[lo] + s_kept[lo] + (p - s_padpre[lo])] = -1;
    }
  }
  for (long long i0 = beg; i0 < end; i0 += 32) {
    const long long i = i0 + lane;
    const bool valid = i < end;
    const int e = valid ? static_cast<int>(s_sel[i]) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank_in = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0) {
      const int rank = hist[w][e] + rank_in;
      if (rank < s_kept[e]) {
        const int pos = s_bstart[e] + rank;
        o.bin_ids[pos] = e;
        o.indices[pos] = static_cast<int32_t>(i);
        const int row = s_pstart[e] + rank;
        if (write_rows) o.row_asg[row] = static_cast<int32_t>(i);
        if (o.asg_row) o.asg_row[i] = row;
      } else if (o.asg_row) {
        o.asg_row[i] = -1;
      }
    } else if (valid && o.asg_row) {
      o.asg_row[i] = -1;
    }
    __syncwarp();
    if (e >= 0 && lane == 31 - __clz(peers)) hist[w][e] += __popc(peers);
    __syncwarp();
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

long long unit_size(long long A) {
  // at most 256 units (the workspace bound); at least 64 assignments (two
  // warp-steps) per unit, so mid-size problems spread over many warps
  long long U = (A + 255) / 256;
  if (U < 64) U = 64;
  return (U + 31) / 32 * 32;
}

}  // namespace

long long route_workspace_bytes(long long A, int E) {
  const long long U = unit_size(A);
  const long long units = (A + U - 1) / U;
  return (units > 0 ? units : 1) * E * 4;
}

template <typename Kern, typename... Args>
static int launch_pdl(Kern kern, int grid, int block, int smem, cudaStream_t st, Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...) == cudaSuccess ? kStatusOk : kStatusCuda;
}

template <typename S>
static int route_impl(const S* sel, long long A, int E, int bs, int mode, const RouteOut& o,
                      void* ws, long long ws_bytes, cudaStream_t st) {
  if (A <= kSmallMaxA) {
    // the kernel's shared-memory limit, raised once per device (callers may be
    // on several host threads)
    static bool attr_set[64] = {};
    static std::mutex attr_mu;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return kStatusCuda;
    {
      std::lock_guard<std::mutex> lock(attr_mu);
      if (!attr_set[dev]) {
        if (cudaFuncSetAttribute(route_small_kernel<S>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kSmallMaxA * 2)) != cudaSuccess)
          return kStatusCuda;
        attr_set[dev] = true;
      }
    }
    const int rc = launch_pdl(route_small_kernel<S>, 1, kSmallWarps * 32,
                              static_cast<int>(A * 2), st, sel, A, E, bs, mode, o);
    if (rc != kStatusOk) return rc;
    return cudaPeekAtLastError() == cudaSuccess ? kStatusOk : kStatusCuda;
  }
  const long long U = unit_size(A);
  const long long units = (A + U - 1) / U;
  if (ws_bytes < route_workspace_bytes(A, E)) return kStatusBadArg;
  int32_t* w = static_cast<int32_t*>(ws);
  const int blocks = static_cast<int>((units + kWarpsPerBlock - 1) / kWarpsPerBlock);
  int rc = launch_pdl(route_count_kernel<S>, blocks, kWarpsPerBlock * 32, 0, st, sel, A, E, U, units,
                      w, o.status);
  if (rc == kStatusOk)
    rc = launch_pdl(route_scan_scatter_kernel<S>, blocks, kWarpsPerBlock * 32, 0, st, sel, A, E,
                    bs, mode, U, units, static_cast<const int32_t*>(w), o);
  if (rc != kStatusOk) return rc;
  return cudaPeekAtLastError() == cudaSuccess ? kStatusOk : kStatusCuda;
}

int route(const void* sel, int sel_is_int64, long long A, int E, int bs, int mode,
          int32_t* bin_ids, int32_t* indices, int32_t* tpe, int32_t* bins, int32_t* padded_bins,
          int32_t* tok_off, int32_t* ptpe, int32_t* row_asg, long long p_cap, int32_t* asg_row,
          void* ws, long long ws_bytes, int* status, cudaStream_t st) {
  if (E <= 0 || E > kMaxE || A < 0 || bs <= 0 || mode < 0 || mode > 2) return kStatusBadArg;
  if (!tpe || !bins || !padded_bins || !tok_off || !ptpe) return kStatusBadArg;
  if (A > 0 && (!sel || !bin_ids || !indices)) return kStatusBadArg;
  RouteOut o{bin_ids, indices, tpe, bins, padded_bins, tok_off, ptpe, row_asg, p_cap, asg_row, status};
  if (sel_is_int64)
    return route_impl(static_cast<const long long*>(sel), A, E, bs, mode, o, ws, ws_bytes, st);
  return route_impl(static_cast<const int32_t*>(sel), A, E, bs, mode, o, ws, ws_bytes, st);
}

// ---- routing without caller-provided scratch ------------------------------------
// The per-unit histogram workspace normally comes from the caller.  This
// variant keeps it in a file-scope device array instead, so it can serve
// callers that cannot allocate device memory.  The array is sized for the
// largest workspace route() can ask for (at most 256 units x 256 experts of
// int32 = 256 KiB); every GPU that loads the library holds it until exit.
// Nothing in it has to start at zero: the count phase writes every entry the
// later phases read.  Every call on a device shares that device's copy and it
// keeps the last call's contents, so two calls whose kernels overlap on the
// same GPU (e.g. issued on different streams) race on it.
namespace {
constexpr long long kRouteScratchInts = 256LL * kMaxE;
constexpr int kMaxDevices = 64;
}  // namespace

static __device__ __align__(256) int32_t g_route_scratch[kRouteScratchInts];

// Device address of g_route_scratch on the current device.  Host code cannot
// use the array's name as a device pointer, so the address is looked up with
// cudaGetSymbolAddress once per device (with that device current) and cached.
static void* route_scratch_address(int* err) {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = kStatusCuda;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_route_scratch) != cudaSuccess || p == nullptr) {
      *err = kStatusCuda;
      return nullptr;
    }
    addr[dev] = p;
  }
  return addr[dev];
}

int route_static_scratch(const void* sel, int sel_is_int64, long long A, int E, int bs, int mode,
                         int32_t* bin_ids, int32_t* indices, int32_t* tpe, int32_t* bins,
                         int32_t* padded_bins, int32_t* tok_off, int32_t* ptpe, int32_t* row_asg,
                         long long p_cap, int32_t* asg_row, int* status, cudaStream_t st) {
  if (E <= 0 || E > kMaxE || A < 0) return kStatusBadArg;
  const long long need = route_workspace_bytes(A, E);
  // unit_size() keeps the unit count <= 256 and E <= kMaxE was checked above,
  // so `need` never exceeds the array today (256 units x kMaxE ints); the check
  // stays as a guard should either bound change
  if (need > kRouteScratchInts * 4) return kStatusCapacity;
  int err = kStatusOk;
  void* ws = route_scratch_address(&err);
  if (ws == nullptr) return err;
  return route(sel, sel_is_int64, A, E, bs, mode, bin_ids, indices, tpe, bins, padded_bins,
               tok_off, ptpe, row_asg, p_cap, asg_row, ws, need, status, st);
}

}  // namespace moe
