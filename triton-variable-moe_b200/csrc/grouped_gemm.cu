// Persistent tcgen05 grouped GEMM: kernel template and host launcher.
// The six reference GEMM kernels (triton_moe/kernels/grouped_gemm.py:212-368,
// 480-583, 654-802, 805-967, 970-1063, 1066-1162) are all instances of this
// one engine; they differ only in operand major-ness, in which metadata array
// supplies each problem dimension, and in the epilogue.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <type_traits>

#include "grouped_gemm.cuh"
#include "moe_internal.h"
#include "sm100_ptx.cuh"

namespace moe {

namespace {

constexpr int BM = 128;   // UMMA M: one TMEM lane per output row
constexpr int BK = 64;    // k-block: one 128-byte swizzle row of bf16
constexpr int UK = 16;    // K per tcgen05.mma (kind::f16)
constexpr int kThreads = 192;

template <int BN>
struct Cfg {
  static constexpr int kStages = (BN == 256) ? 4 : 6;
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;  // double-buffered fp32 accumulator
  static constexpr int kEpiBytes = 4 * 32 * 128;  // per epilogue warp: 32 rows x 64 bf16
  static constexpr int kSmemBytes =
      1024 /*align slack*/ + kStages * kStageBytes + kEpiBytes + 256 /*barriers*/;
};

struct GroupTable {
  int prefix[kMaxGroups + 1];
  int M[kMaxGroups], N[kMaxGroups], K[kMaxGroups];
  int am[kMaxGroups], ak[kMaxGroups], bn[kMaxGroups], bk[kMaxGroups];
  int dm[kMaxGroups], dn[kMaxGroups];
};

__device__ __forceinline__ int dim_value(int src, int e, const GroupedGemmDesc& g) {
  if (src == DIM_TOKENS) return g.tok_off[e + 1] - g.tok_off[e];
  if (src == DIM_WIDTH) return g.w_off[e + 1] - g.w_off[e];
  return g.cdim;
}
__device__ __forceinline__ int base_value(int src, int e, const GroupedGemmDesc& g) {
  if (src == BASE_TOK) return g.tok_off[e];
  if (src == BASE_WOFF) return g.w_off[e];
  return 0;
}

template <typename T>
struct Cvt;
template <>
struct Cvt<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float round(float a) {
    return __bfloat162float(__float2bfloat16_rn(a));
  }
  static __device__ __forceinline__ void unpack(uint32_t u, float& a, float& b) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&u);
    float2 f = __bfloat1622float2(h);
    a = f.x;
    b = f.y;
  }
};
template <>
struct Cvt<__half> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float round(float a) {
    return __half2float(__float2half_rn(a));
  }
  static __device__ __forceinline__ void unpack(uint32_t u, float& a, float& b) {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    float2 f = __half22float2(h);
    a = f.x;
    b = f.y;
  }
};

template <int BN>
__device__ __forceinline__ void decode_tile(const GroupTable& tb, int E, int t, int& e,
                                            int& m0, int& n0) {
  int lo = 0, hi = E - 1;  // find e with prefix[e] <= t < prefix[e+1]
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (tb.prefix[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  e = lo;
  const int local = t - tb.prefix[e];
  const int ntn = (tb.N[e] + BN - 1) / BN;
  m0 = (local / ntn) * BM;
  n0 = (local % ntn) * BN;
}

template <int BN, bool A_MN, bool B_MN, int EPI, typename T>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const GroupedGemmDesc g) {
  using C = Cfg<BN>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;                      // S stages of A
  uint8_t* sB = smem + S * C::kABytes;     // S stages of B
  uint8_t* sEpi = smem + S * C::kStageBytes;  // epilogue staging, 4 KB per warp
  uint64_t* bars = reinterpret_cast<uint64_t*>(sEpi + C::kEpiBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* acc_full = bars + 2 * S;
  uint64_t* acc_empty = bars + 2 * S + 2;
  uint64_t* drain = bars + 2 * S + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);

  __shared__ GroupTable tb;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  // Everything above touched only this CTA's own resources; from here on the
  // kernel reads and writes global memory that earlier kernels in the stream
  // produce or consume, so wait for them (programmatic dependent launch).
  griddep_wait();
  if (warp == 2) {
    // Per-expert geometry and the tile prefix table: lane L owns a contiguous
    // chunk of experts, then a warp scan turns chunk sums into offsets.
    const int E = g.E;
    const int per = (E + 31) / 32;
    const int beg = lane * per;
    const int end = min(E, beg + per);
    int sum = 0;
    for (int e = beg; e < end; ++e) {
      int M = dim_value(g.m_src, e, g);
      if (g.m_src == DIM_TOKENS && g.tok_cnt != nullptr) M = min(M, g.tok_cnt[e]);
      M = max(M, 0);
      const int N = dim_value(g.n_src, e, g);
      const int K = dim_value(g.k_src, e, g);
      tb.M[e] = M;
      tb.N[e] = N;
      tb.K[e] = max(K, 0);
      tb.am[e] = base_value(g.a_m_base, e, g);
      tb.ak[e] = base_value(g.a_k_base, e, g);
      tb.bn[e] = base_value(g.b_n_base, e, g);
      tb.bk[e] = base_value(g.b_k_base, e, g);
      tb.dm[e] = base_value(g.d_m_base, e, g);
      tb.dn[e] = base_value(g.d_n_base, e, g);
      // TMA needs 16-byte aligned inner coordinates and the MMA consumes K in
      // steps of 16: reject (and skip) any expert whose geometry breaks that.
      const bool bad = (K % 16) != 0 || (g.n_src == DIM_WIDTH && N % 16 != 0) ||
                       (g.m_src == DIM_WIDTH && M % 16 != 0) || (tb.bn[e] % 8) != 0 ||
                       (tb.bk[e] % 8) != 0 || (tb.dn[e] % 8) != 0;
      if (bad && g.status != nullptr) atomicExch(g.status, kStatusBadArg);
      const int tiles =
          (!bad && M > 0 && N > 0) ? ((M + BM - 1) / BM) * ((N + BN - 1) / BN) : 0;
      tb.prefix[e] = sum;  // chunk-local exclusive prefix for now
      sum += tiles;
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int excl = incl - sum;
    for (int e = beg; e < end; ++e) tb.prefix[e] += excl;
    if (lane == 31) tb.prefix[E] = incl;
  }
  __syncthreads();
  tc_fence_after();
  // The next kernel may start its own prologue now; it waits for this grid's
  // completion before touching memory.
  griddep_launch_dependents();
  const uint32_t tmem_base = *tmem_slot;
  const int E = g.E;
  const int total = tb.prefix[E];

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        int e, m0, n0;
        decode_tile<BN>(tb, E, t, e, m0, n0);
        const int K = tb.K[e];
        const int nkb = (K + BK - 1) / BK;
        const int am = tb.am[e] + m0, ak = tb.ak[e];
        const int bn = tb.bn[e] + n0, bk = tb.bk[e];
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, &abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
          uint8_t* a_dst = sA + stage * C::kABytes;
          uint8_t* b_dst = sB + stage * C::kBBytes;
          const int kc = kb * BK;
          if constexpr (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_2d(a_dst + j * 8192, &tmA, &full[stage], am + 64 * j, ak + kc);
          } else {
            tma_load_2d(a_dst, &tmA, &full[stage], ak + kc, am);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(b_dst + j * 8192, &tmB, &full[stage], bn + 64 * j, bk + kc);
          } else {
            tma_load_2d(b_dst, &tmB, &full[stage], bk + kc, bn);
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc =
          idesc_f16(BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0, std::is_same<T, __half>::value ? 1 : 0);
      int stage = 0;
      uint32_t phase = 0;
      int buf = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int e, m0, n0;
        decode_tile<BN>(tb, E, t, e, m0, n0);
        const int K = tb.K[e];
        const int nkb = (K + BK - 1) / BK;
        if (!mbar_wait(&acc_empty[buf], acc_phase ^ 1, &abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&full[stage], phase, &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * C::kABytes);
          const uint32_t b_addr = smem_u32(sB + stage * C::kBBytes);
          const int kvalid = min(BK, K - kb * BK);
          const int nk = kvalid / UK;
          for (int kk = 0; kk < nk; ++kk) {
            uint64_t ad, bd;
            if constexpr (A_MN) ad = smem_desc_sw128(a_addr + kk * 2048, 8192, 1024);
            else ad = smem_desc_sw128(a_addr + kk * 32, 16, 1024);
            if constexpr (B_MN) bd = smem_desc_sw128(b_addr + kk * 2048, 8192, 1024);
            else bd = smem_desc_sw128(b_addr + kk * 32, 16, 1024);
            tc_mma_f16(d_tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&empty[stage]);  // smem stage free once these MMAs retire
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if (nkb > 0) tc_commit(&acc_full[buf]);
        else mbar_arrive(&acc_full[buf]);
        buf ^= 1;
        if (buf == 0) acc_phase ^= 1;
      }
      // Make sure no MMA is still in flight before TMEM is released.
      tc_commit(drain);
      mbar_wait(drain, 0, &abort_flag);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // Each warp owns 32 accumulator rows (its TMEM lane quarter).  Results are
    // produced one 64-column slab at a time: every lane converts its own row
    // into a 32 x 128 B staging tile (16-byte chunks XOR-swizzled by row, so
    // the row-per-lane writes and the row-major reads are bank-conflict free),
    // then the warp stores the slab row-major, four full 128-byte rows per
    // instruction.
    const int q = warp & 3;
    uint8_t* stg = sEpi + q * 4096;
    int buf = 0;
    uint32_t acc_phase = 0;
    T* D = reinterpret_cast<T*>(g.d);
    T* AUX = reinterpret_cast<T*>(g.aux);
    const int rsub = lane >> 3;  // row within a 4-row group for the row-major phase
    const int csub = lane & 7;   // 16-byte chunk within a 128-byte row
    auto stg_chunk = [&](int row, int chunk) -> uint4* {
      return reinterpret_cast<uint4*>(stg + row * 128 + ((chunk ^ (row & 7)) << 4));
    };
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      int e, m0, n0;
      decode_tile<BN>(tb, E, t, e, m0, n0);
      const int M = tb.M[e], N = tb.N[e], K = tb.K[e];
      if (!mbar_wait(&acc_full[buf], acc_phase, &abort_flag)) break;
      tc_fence_after();
      const int rbase = m0 + q * 32;            // group row of this warp's first row
      const int rows_ok = min(32, M - rbase);   // may be <= 0
      const long long grow0 = static_cast<long long>(tb.dm[e]) + rbase;
      const int gcol0 = tb.dn[e] + n0;
      const int ncols = min(BN, N - n0);
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN);
      // row-major store of the staged slab (rows beyond the expert and columns
      // beyond its width are skipped); all shared loads first, then the stores
      auto store_slab = [&](T* dst, long long ld, int s, int cvalid) {
        uint4 sv[8];
#pragma unroll
        for (int it = 0; it < 8; ++it) sv[it] = *stg_chunk(it * 4 + rsub, csub);
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int row = it * 4 + rsub;
          if (row < rows_ok && csub * 8 < cvalid)
            *reinterpret_cast<uint4*>(dst + (grow0 + row) * ld + gcol0 + s + csub * 8) = sv[it];
        }
      };
#pragma unroll 1
      for (int s = 0; s < ncols; s += 64) {
        const int cvalid = min(64, ncols - s);
        float v[64];
        if (K > 0) {
          tmem_ld32(tbase + s, *reinterpret_cast<float(*)[32]>(&v[0]));
          if (cvalid > 32) tmem_ld32(tbase + s + 32, *reinterpret_cast<float(*)[32]>(&v[32]));
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i) v[i] = 0.f;
        }
        if constexpr (EPI == EPI_STORE) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 o;
            uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
            for (int i = 0; i < 4; ++i) op[i] = Cvt<T>::pack(v[j * 8 + 2 * i], v[j * 8 + 2 * i + 1]);
            *stg_chunk(lane, j) = o;
          }
          __syncwarp();
          store_slab(D, g.ldd, s, cvalid);
          __syncwarp();
        } else if constexpr (EPI == EPI_RELU2) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 o;
            uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              v[j * 8 + 2 * i] = fmaxf(v[j * 8 + 2 * i], 0.f);
              v[j * 8 + 2 * i + 1] = fmaxf(v[j * 8 + 2 * i + 1], 0.f);
              op[i] = Cvt<T>::pack(v[j * 8 + 2 * i], v[j * 8 + 2 * i + 1]);
            }
            *stg_chunk(lane, j) = o;
          }
          __syncwarp();
          store_slab(AUX, g.ld_aux, s, cvalid);
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 o;
            uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float a = v[j * 8 + 2 * i], b = v[j * 8 + 2 * i + 1];
              op[i] = Cvt<T>::pack(a * a, b * b);
            }
            *stg_chunk(lane, j) = o;
          }
          __syncwarp();
          store_slab(D, g.ldd, s, cvalid);
          __syncwarp();
        } else {  // EPI_DACT: stage pre (row-major, coalesced), combine per row
          uint4 pv[8];  // all eight loads in flight before any shared store
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int row = it * 4 + rsub;
            pv[it] = make_uint4(0, 0, 0, 0);
            if (row < rows_ok && csub * 8 < cvalid)
              pv[it] = __ldg(reinterpret_cast<const uint4*>(AUX + (grow0 + row) * g.ld_aux +
                                                            gcol0 + s + csub * 8));
          }
#pragma unroll
          for (int it = 0; it < 8; ++it) *stg_chunk(it * 4 + rsub, csub) = pv[it];
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint4 p = *stg_chunk(lane, j);
            const uint32_t* pp = reinterpret_cast<const uint32_t*>(&p);
            uint4 o;
            uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              float p0, p1;
              Cvt<T>::unpack(pp[i], p0, p1);
              const float g0 = Cvt<T>::round(v[j * 8 + 2 * i]);
              const float g1 = Cvt<T>::round(v[j * 8 + 2 * i + 1]);
              op[i] = Cvt<T>::pack(p0 > 0.f ? g0 * 2.0f * p0 : 0.f, p1 > 0.f ? g1 * 2.0f * p1 : 0.f);
            }
            *stg_chunk(lane, j) = o;
          }
          __syncwarp();
          store_slab(D, g.ldd, s, cvalid);
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      buf ^= 1;
      if (buf == 0) acc_phase ^= 1;
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
  if (threadIdx.x == 0 && abort_flag && g.status != nullptr) atomicExch(g.status, kStatusTimeout);
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D row-major tensor [outer, inner] with row stride `ld` elements, 128-byte
// swizzled boxes of box_inner x box_outer elements.
int make_tmap(CUtensorMap* tm, const void* base, int is_f16, long long inner, long long outer,
              long long ld, int box_inner, int box_outer) {
  auto fn = encode_fn();
  if (!fn) return kStatusCuda;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld * 2) % 16 != 0) return kStatusBadArg;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(tm, is_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                  2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kStatusOk : kStatusBadArg;
}

template <int BN, bool A_MN, bool B_MN, int EPI, typename T>
int launch_inst(const CUtensorMap& ta, const CUtensorMap& tbm, const GroupedGemmDesc& g,
                int grid, cudaStream_t st) {
  auto kern = grouped_gemm_kernel<BN, A_MN, B_MN, EPI, T>;
  constexpr int smem = Cfg<BN>::kSmemBytes;
  static bool attr_set[64] = {};  // per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) !=
            cudaSuccess)
      return kStatusCuda;
    attr_set[dev] = true;
  }
  // Programmatic dependent launch: this grid's prologue (barrier init, TMEM
  // allocation, descriptor prefetch) overlaps the tail of the previous kernel.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, ta, tbm, g) != cudaSuccess) return kStatusCuda;
  return cudaPeekAtLastError() == cudaSuccess ? kStatusOk : kStatusCuda;
}

template <int BN, int EPI, typename T>
int dispatch_major(const GemmOperands& op, const CUtensorMap& ta, const CUtensorMap& tbm,
                   const GroupedGemmDesc& g, int grid, cudaStream_t st) {
  if (!op.a_mn && !op.b_mn) return launch_inst<BN, false, false, EPI, T>(ta, tbm, g, grid, st);
  if (!op.a_mn && op.b_mn) return launch_inst<BN, false, true, EPI, T>(ta, tbm, g, grid, st);
  if (op.a_mn && op.b_mn) return launch_inst<BN, true, true, EPI, T>(ta, tbm, g, grid, st);
  return kStatusUnsupported;  // MN-major A with K-major B is not used by any MoE GEMM
}

template <int EPI, typename T>
int dispatch_bn(const GemmOperands& op, int bn, const CUtensorMap& ta, const CUtensorMap& tbm,
                const GroupedGemmDesc& g, int grid, cudaStream_t st) {
  if (bn == 256) return dispatch_major<256, EPI, T>(op, ta, tbm, g, grid, st);
  return dispatch_major<128, EPI, T>(op, ta, tbm, g, grid, st);
}

}  // namespace

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

int run_grouped_gemm(const GemmOperands& op, const GroupedGemmDesc& g, int epi, int is_f16,
                     cudaStream_t st) {
  if (g.E <= 0) return kStatusOk;
  if (g.E > kMaxGroups) return kStatusUnsupported;
  if (op.a_rows <= 0 || op.a_cols <= 0 || op.b_rows <= 0 || op.b_cols <= 0)
    return kStatusBadArg;
  const int bn = op.bn == 256 ? 256 : 128;
  CUtensorMap ta, tbm;
  int s;
  // A is [a_rows, a_cols] row-major.  K-major A: rows are M, columns are K.
  // MN-major A: rows are K, columns are M.
  if (op.a_mn) s = make_tmap(&ta, op.a, is_f16, op.a_cols, op.a_rows, op.lda, 64, 64);
  else s = make_tmap(&ta, op.a, is_f16, op.a_cols, op.a_rows, op.lda, 64, BM);
  if (s) return s;
  if (op.b_mn) s = make_tmap(&tbm, op.b, is_f16, op.b_cols, op.b_rows, op.ldb, 64, 64);
  else s = make_tmap(&tbm, op.b, is_f16, op.b_cols, op.b_rows, op.ldb, 64, bn);
  if (s) return s;
  const int grid = op.grid > 0 ? op.grid : num_sms();
  if (is_f16) {
    if (epi == EPI_STORE) return dispatch_bn<EPI_STORE, __half>(op, bn, ta, tbm, g, grid, st);
    if (epi == EPI_RELU2) return dispatch_bn<EPI_RELU2, __half>(op, bn, ta, tbm, g, grid, st);
    return dispatch_bn<EPI_DACT, __half>(op, bn, ta, tbm, g, grid, st);
  }
  if (epi == EPI_STORE) return dispatch_bn<EPI_STORE, __nv_bfloat16>(op, bn, ta, tbm, g, grid, st);
  if (epi == EPI_RELU2) return dispatch_bn<EPI_RELU2, __nv_bfloat16>(op, bn, ta, tbm, g, grid, st);
  return dispatch_bn<EPI_DACT, __nv_bfloat16>(op, bn, ta, tbm, g, grid, st);
}

}  // namespace moe
