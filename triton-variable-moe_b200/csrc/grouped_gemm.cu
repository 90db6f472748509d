// Persistent tcgen05 grouped GEMM: kernel and host launcher.
//
// The six reference GEMM kernels (triton_moe/kernels/grouped_gemm.py:212-368,
// 480-583, 654-802, 805-967, 970-1063, 1066-1162) are all problems of this
// one engine; they differ only in operand major-ness, in which metadata array
// supplies each problem dimension, in the N tile and in the epilogue -- all
// runtime properties of a problem.  One launch runs up to kMaxProblems
// independent problems over a single tile list (the backward's dIntermediate
// + dW2 pair and dX + dW1 pair), so the SMs stay busy across the boundary
// between them and a launch boundary disappears.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>
#include <type_traits>

#include "grouped_gemm.cuh"
#include "moe_internal.h"
#include "sm100_ptx.cuh"
#include "trace.cuh"

namespace moe {

namespace {

constexpr int BM = 128;  // UMMA M: one TMEM lane per output row
constexpr int BN_MAX = 256;
#ifndef MOE_EPI_WARPS
#define MOE_EPI_WARPS 4
#endif
// Epilogue warps: 4 (one per TMEM lane quarter) or 8 (two per quarter, each
// taking half of a tile's column slabs).  8 take 32 KB more staging memory, so
// the ring has 3 stages instead of 4 at N tile 256; measured slower at the c3
// and c4 shapes (c3 GEMM step 88 vs 82 us), hence 4.
constexpr int kEpiWarps = MOE_EPI_WARPS;
static_assert(kEpiWarps == 4 || kEpiWarps == 8, "4 or 8 epilogue warps");
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kMaxStages = 8;
constexpr int kABytes = BM * 128;        // 16 KB: 128 rows of one 128-byte k-block
constexpr int kSmemMax = 227 * 1024;     // dynamic shared memory per CTA on sm_100
// Epilogue staging per warp: two 32-row x 128-byte slabs (a slab is rewritten
// while the other's TMA store reads it), or one in the ticket-order build,
// whose long tiles leave the epilogue time to spare and which needs the 16 KB
// for its ring (4 stages of 48 KB beside a large slot table).
constexpr int epi_slabs(bool dyn) { return dyn ? 1 : 2; }
constexpr int epi_bytes(bool dyn) { return kEpiWarps * epi_slabs(dyn) * 32 * 128; }
constexpr int kTmemCols = 2 * BN_MAX;    // double-buffered fp32 accumulator
constexpr int kBarBytes = 640;            // mbarriers, TMEM address, abort flag, tile queue
constexpr int kTileQ = 8;                 // tile queue entries (producer -> MMA / epilogue)
constexpr int kDynMinTiles = 8;           // tiles per unit from which tiles are taken by ticket

struct Problem {
  GroupedGemmDesc g;
  int a_mn, b_mn, epi, bn;
  int tile_n;  // output columns per tile: bn, or bn / 2 for SwiGLU (gate + up halves)
  int d_tma;   // tmD is valid: full slabs leave through TMA stores
};

struct MultiParams {
  CUtensorMap tmA[kMaxProblems];
  CUtensorMap tmB[kMaxProblems];
  CUtensorMap tmD[kMaxProblems];  // epilogue output, 32-row x 128-byte boxes
  CUtensorMap tmX[kMaxProblems];  // epilogue aux (pre-activation), same boxes
  CUtensorMap tmY[kMaxProblems];  // epilogue aux2 (SwiGLU up), same boxes
  Problem pr[kMaxProblems];
  int nprob;
  int stages;       // stages in the ring (depends on the largest N tile)
  int stage_bytes;  // A tile + largest B tile
  int smem_bytes;   // dynamic shared memory of the launch
  unsigned long long wait_ns;  // limit of every device-side wait (ns)
  int* sched;  // tile-ticket counter (zero between launches), or null: round-robin tiles
};

// Per (problem, expert) slot: tile prefix, extents and the two offsets every
// coordinate base is made of (token offset, weight offset).  Lives in dynamic
// shared memory behind the barriers, sized for the launch's slot count.
struct Table {
  int* prefix;  // [nge + 1]
  int *M, *N, *K, *tok, *wof;  // [nge] each
  int* mtp;  // [nge] first row block (of BMT rows) of each problem-0 slot
};
__host__ __device__ constexpr int table_bytes(int nge) { return (7 * nge + 1) * 4; }

__device__ __forceinline__ int slot_base(int src, const Table& tb, int slot) {
  if (src == BASE_TOK) return tb.tok[slot];
  if (src == BASE_WOFF) return tb.wof[slot];
  return 0;
}

__device__ __forceinline__ int dim_value(int src, int e, const GroupedGemmDesc& g) {
  if (src == DIM_TOKENS) return g.tok_off[e + 1] - g.tok_off[e];
  if (src == DIM_WIDTH) return g.w_off[e + 1] - g.w_off[e];
  if (src == DIM_HALF_WIDTH) return (g.w_off[e + 1] - g.w_off[e]) / 2;
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

template <>
struct Cvt<float> {
  static __device__ __forceinline__ float round(float a) { return a; }
};

// Per element type: bytes, elements per 128-byte swizzle row (the k-block),
// elements per MMA K step (32 bytes), elements per 16-byte chunk, and the
// tcgen05 operand format code.
template <typename T>
struct Elem {
  static constexpr int ES = sizeof(T);
  static constexpr int BKE = 128 / ES;
  static constexpr int UKE = 32 / ES;
  static constexpr int EPC = 16 / ES;
  static constexpr int FMT = std::is_same<T, float>::value ? 2 : (std::is_same<T, __half>::value ? 0 : 1);
};

template <typename T>
__device__ __forceinline__ uint4 pack_chunk(const float* v) {
  uint4 o;
  uint32_t* op = reinterpret_cast<uint32_t*>(&o);
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) op[i] = __float_as_uint(v[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) op[i] = Cvt<T>::pack(v[2 * i], v[2 * i + 1]);
  }
  return o;
}
template <typename T>
__device__ __forceinline__ void unpack_chunk(const uint4& u, float* v) {
  const uint32_t* up = reinterpret_cast<const uint32_t*>(&u);
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(up[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) Cvt<T>::unpack(up[i], v[2 * i], v[2 * i + 1]);
  }
}

struct Tile {
  int p, e, m0, n0, slot;
};

template <int BMT>
__device__ __forceinline__ Tile decode_tile(const Table& tb, const MultiParams& P, int nge,
                                            int t) {
  int lo = 0, hi = nge - 1;  // last (problem, expert) slot with prefix <= t
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tb.prefix[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  Tile r;
  r.p = lo < P.pr[0].g.E ? 0 : 1;  // slots are problem 0's experts, then problem 1's
  r.e = lo - (r.p ? P.pr[0].g.E : 0);
  r.slot = lo;
  const int bn = P.pr[r.p].tile_n;
  const int local = t - tb.prefix[lo];
  const int ntn = (tb.N[lo] + bn - 1) / bn;
  r.m0 = (local / ntn) * BMT;
  r.n0 = (local % ntn) * bn;
  return r;
}

// Compile-time operand configuration of a problem slot: bit 0 = A MN-major,
// bit 1 = B MN-major, bit 2 = N tile 256 (else 128), bit 4 = the SwiGLU
// epilogue is compiled in (only the up projection's kernels carry it).
constexpr int kCfgSwiglu = 16;
constexpr int cfg_of(int a_mn, int b_mn, int bn, bool swiglu = false) {
  return a_mn | (b_mn << 1) | ((bn == 256) << 2) | (swiglu ? kCfgSwiglu : 0);
}

// Producer side of one tile: stream its k-blocks into the smem ring.  A tile
// is 128 rows (A) / NT rows (B) of one 128-byte swizzle row of K each; an
// MN-major operand arrives as 128-byte-wide MN blocks, one box each.
// With a CTA pair (CG = 2) each CTA loads its own 128 rows of A and its half
// (NT / 2 rows) of B; am / bn are already offset to this CTA's share.
template <int CFG, typename T, int CG>
__device__ __forceinline__ bool produce_tile(uint8_t* ring, int SB, int S, uint64_t* full,
                                             uint64_t* empty, volatile int* abort_flag,
                                             uint64_t wait_ns, const void* tA,
                                             const void* tB, int nkb, int am, int ak, int bn,
                                             int bk, int& stage, uint32_t& phase, int up_shift,
                                             int& issued) {
  constexpr bool A_MN = CFG & 1, B_MN = (CFG >> 1) & 1;
  constexpr int NT = ((CFG & 4) ? 256 : 128) / CG;  // B rows this CTA loads
  constexpr int BKE = Elem<T>::BKE;
  constexpr uint32_t bytes = kABytes + NT * 128;
  for (int kb = 0; kb < nkb; ++kb) {
    if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, wait_ns)) return false;
    MOE_TRACE_KB(issued, 0);
    mbar_arrive_expect_tx(&full[stage], bytes);
    uint8_t* a_dst = ring + stage * SB;
    uint8_t* b_dst = a_dst + kABytes;
    const int kc = kb * BKE;
    if constexpr (A_MN) {
#pragma unroll
      for (int j = 0; j < BM / BKE; ++j)
        tma_load_2d(a_dst + j * BKE * 128, tA, &full[stage], am + BKE * j, ak + kc);
    } else {
      tma_load_2d(a_dst, tA, &full[stage], ak + kc, am);
    }
    if constexpr (B_MN) {
      // SwiGLU (up_shift != 0): the second half of the tile's columns comes
      // from the expert's up block, up_shift columns further
#pragma unroll
      for (int j = 0; j < NT / BKE; ++j)
        tma_load_2d(b_dst + j * BKE * 128, tB, &full[stage],
                    bn + BKE * j + (j >= NT / BKE / 2 ? up_shift : 0), bk + kc);
    } else {
      tma_load_2d(b_dst, tB, &full[stage], bk + kc, bn);
    }
    ++issued;
    if (++stage == S) {
      stage = 0;
      phase ^= 1;
    }
  }
  return true;
}

// After an abort: wait (bounded, ignoring the abort flag) until the stages
// this producer loaded last have landed, so that no TMA write into shared
// memory is in flight when the CTA exits.  (stage, phase) is the producer's
// next write; `issued` counts the k-blocks it loaded.
__device__ __forceinline__ void drain_loads(uint64_t* full, int S, int stage, uint32_t phase,
                                            int issued, uint64_t wait_ns) {
  int no_abort = 0;
  for (int j = 0; j < S && j < issued; ++j) {
    if (stage == 0) {
      stage = S - 1;
      phase ^= 1;
    } else {
      --stage;
    }
    mbar_wait(&full[stage], phase, &no_abort, wait_ns);
  }
}

// MMA side of one tile: issue its k-blocks into the TMEM accumulator.
// With a CTA pair (CG = 2) this runs on the even CTA only: a stage is used
// once both CTAs' halves have landed (`peer_full` is arrived on by the odd
// CTA's relay), one M = 256 MMA covers both halves, and the stage is released
// in both CTAs.
template <int CFG, typename T, int CG>
__device__ __forceinline__ bool mma_tile(uint8_t* ring, int SB, int S, uint64_t* full,
                                         uint64_t* peer_full, uint64_t* empty,
                                         volatile int* abort_flag, uint64_t wait_ns,
                                         uint32_t d_tmem, int K,
                                         int nkb, int& stage, uint32_t& phase, int& seen) {
  constexpr int A_MN = CFG & 1, B_MN = (CFG >> 1) & 1;
  constexpr int NT = (CFG & 4) ? 256 : 128;
  constexpr int BKE = Elem<T>::BKE, UKE = Elem<T>::UKE;
  constexpr uint32_t idesc = idesc_mma(BM * CG, NT, A_MN, B_MN, Elem<T>::FMT);
  // K-major: the next K step is 32 bytes further along the swizzled row.
  // MN-major: it is UKE rows (of 128 bytes) further; MN blocks are LBO apart.
  constexpr uint32_t a_step = A_MN ? UKE * 128u : 32u, a_lbo = A_MN ? BKE * 128u : 16u;
  constexpr uint32_t b_step = B_MN ? UKE * 128u : 32u, b_lbo = B_MN ? BKE * 128u : 16u;
  // MN-major fp32 tiles use the 32-byte-granular swizzle: 4-row K groups.
  constexpr bool kW = sizeof(T) == 4;
  constexpr uint32_t a_sbo = (A_MN && kW) ? 512u : 1024u, a_lay = (A_MN && kW) ? 1u : 2u;
  constexpr uint32_t b_sbo = (B_MN && kW) ? 512u : 1024u, b_lay = (B_MN && kW) ? 1u : 2u;
  for (int kb = 0; kb < nkb; ++kb) {
    if (!mbar_wait(&full[stage], phase, abort_flag, wait_ns)) return false;
    if constexpr (CG == 2)
      if (!mbar_wait_cluster(&peer_full[stage], phase, abort_flag, wait_ns)) return false;
    MOE_TRACE_KB(seen, 1);
    ++seen;
    tc_fence_after();
    const uint32_t a_addr = smem_u32(ring + stage * SB);
    const uint32_t b_addr = a_addr + kABytes;
    const int nk = min(BKE, K - kb * BKE) / UKE;
    for (int kk = 0; kk < nk; ++kk) {
      const uint64_t ad = smem_desc_sw128(a_addr + kk * a_step, a_lbo, a_sbo, a_lay);
      const uint64_t bd = smem_desc_sw128(b_addr + kk * b_step, b_lbo, b_sbo, b_lay);
      const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
      if constexpr (sizeof(T) == 4) tc_mma_tf32<CG>(d_tmem, ad, bd, idesc, acc);
      else tc_mma_f16<CG>(d_tmem, ad, bd, idesc, acc);
    }
    // smem stage free (in both CTAs of a pair) once these MMAs retire
    if constexpr (CG == 2) tc_commit_pair(&empty[stage]);
    else tc_commit(&empty[stage]);
    if (++stage == S) {
      stage = 0;
      phase ^= 1;
    }
  }
  return true;
}

// CG = 2: launched as 2-CTA clusters; the pair computes 256-row tiles with
// cta_group::2 MMAs issued by the even CTA, each CTA holding its 128 rows of
// the accumulator and running its own producer and epilogue.
template <typename T, int CFG0, int CFG1, int CG, bool DYN>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ MultiParams P) {
  constexpr int BMT = BM * CG;  // tile rows
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int S = P.stages;
  const int SB = P.stage_bytes;
  uint8_t* ring = smem;                // stage s: A at s*SB, B at s*SB + kABytes
  uint8_t* sEpi = smem + S * SB;       // epilogue staging, 4 KB slabs per warp
  constexpr int kSlabs = epi_slabs(DYN);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sEpi + epi_bytes(DYN));
  uint64_t* full = bars;
  uint64_t* empty = bars + kMaxStages;
  uint64_t* acc_full = bars + 2 * kMaxStages;
  uint64_t* acc_empty = bars + 2 * kMaxStages + 2;
  uint64_t* drain = bars + 2 * kMaxStages + 4;
  uint64_t* epi_ld = bars + 3 * kMaxStages + 15;  // [epilogue warps][2 slabs]: aux loads
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 13);
  int& abort_flag = *reinterpret_cast<int*>(bars + 2 * kMaxStages + 14);
  uint64_t* peer_full = bars + 2 * kMaxStages + 15;  // [stages], even CTA of a pair
  // tile queue (ticket order only): the producer pushes each tile's index (-1
  // after the last); the MMA issuer (or a pair's relay) and every epilogue
  // warp pop it
  uint64_t* tq_full = bars + 3 * kMaxStages + 15 + 2 * 8;  // after epi_ld's 16 slots
  uint64_t* tq_empty = tq_full + kTileQ;
  int* tq = reinterpret_cast<int*>(tq_empty + kTileQ);
  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
  const int unit = CG == 2 ? static_cast<int>(blockIdx.x) / 2 : static_cast<int>(blockIdx.x);
  const int nunits = CG == 2 ? static_cast<int>(gridDim.x) / 2 : static_cast<int>(gridDim.x);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint64_t wait_ns = P.wait_ns;
  // waits that must complete even after an abort (this CTA's own copies and
  // MMAs in flight) see this flag, which stays 0, and only their time limit
  int no_abort = 0;
  if (threadIdx.x == 0) MOE_TRACE_AT(0);
  // (problem, expert) slots: problem 0's experts, then problem 1's
  const int nge = P.pr[0].g.E + (P.nprob > 1 ? P.pr[1].g.E : 0);
  Table tb;
  tb.prefix = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(bars) + kBarBytes);
  tb.M = tb.prefix + nge + 1;
  tb.N = tb.M + nge;
  tb.K = tb.N + nge;
  tb.tok = tb.K + nge;
  tb.wof = tb.tok + nge;
  tb.mtp = tb.wof + nge;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      mbar_init(&peer_full[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpiWarps * CG);  // one arrival per epilogue warp of the pair
    }
    mbar_init(drain, 1);
    for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&epi_ld[i], 1);
    if constexpr (DYN) {
      for (int i = 0; i < kTileQ; ++i) {
        mbar_init(&tq_full[i], 1);
        mbar_init(&tq_empty[i], 1 + kEpiWarps);
      }
    }
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    for (int p = 0; p < P.nprob; ++p) {
      tma_prefetch_desc(&P.tmA[p]);
      tma_prefetch_desc(&P.tmB[p]);
    }
  }
  if (warp >= 2 && lane == 0 && warp - 2 < P.nprob) {
    if (P.pr[warp - 2].d_tma) tma_prefetch_desc(&P.tmD[warp - 2]);
    if (P.pr[warp - 2].epi == EPI_DACT) tma_prefetch_desc(&P.tmX[warp - 2]);
  }
  if (warp == 1) {
    tmem_alloc<CG>(tmem_slot, kTmemCols);
    tmem_relinquish<CG>();
    tc_fence_before();
  }
  // The slot table reads only the expert offset arrays, which no kernel of the
  // stream writes after the routing: every kernel here lets its dependents
  // launch only after its own programmatic-launch wait, so when this grid
  // starts every kernel before its immediate predecessor has completed, the
  // routing included.  Building the table before this grid's own wait overlaps
  // it with the predecessor's tail.
  if (warp == 2) {
    // Per-(problem, expert) geometry and the tile prefix table: lane L owns a
    // contiguous chunk of slots, then a warp scan turns chunk sums into offsets.
    const int per = (nge + 31) / 32;
    const int beg = lane * per;
    const int end = min(nge, beg + per);
    int sum = 0, msum = 0;
    for (int s = beg; s < end; ++s) {
      const int p = s < P.pr[0].g.E ? 0 : 1;
      const int e = s - (p ? P.pr[0].g.E : 0);
      const GroupedGemmDesc& g = P.pr[p].g;
      int M = 0, N = 0, K = 0, tiles = 0;
      {
        M = dim_value(g.m_src, e, g);
        if (g.m_src == DIM_TOKENS && g.tok_cnt != nullptr) M = min(M, g.tok_cnt[e]);
        M = max(M, 0);
        N = dim_value(g.n_src, e, g);
        K = max(dim_value(g.k_src, e, g), 0);
        // TMA needs 16-byte aligned inner coordinates and the MMA consumes K in
        // steps of 16: reject (and skip) any expert whose geometry breaks that.
        constexpr int kAlign = 16 / static_cast<int>(sizeof(T));  // elements per 16 bytes
        const bool bad = (K % Elem<T>::UKE) != 0 || (g.n_src == DIM_WIDTH && N % 16 != 0) ||
                         (g.m_src == DIM_WIDTH && M % 16 != 0) ||
                         (base_value(g.b_n_base, e, g) % kAlign) != 0 ||
                         (base_value(g.b_k_base, e, g) % kAlign) != 0 ||
                         (base_value(g.d_n_base, e, g) % kAlign) != 0;
        if (bad && g.status != nullptr) atomicExch(g.status, kStatusBadArg);
        const int bn = P.pr[p].tile_n;
        tiles = (!bad && M > 0 && N > 0) ? ((M + BMT - 1) / BMT) * ((N + bn - 1) / bn) : 0;
      }
      tb.M[s] = M;
      tb.N[s] = N;
      tb.K[s] = K;
      tb.tok[s] = g.tok_off[e];
      tb.wof[s] = g.w_off[e];
      tb.prefix[s] = sum;  // chunk-local exclusive prefixes for now
      sum += tiles;
      tb.mtp[s] = msum;
      if (p == 0) msum += (M + BMT - 1) / BMT;
    }
    int incl = sum, mincl = msum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      const int mv = __shfl_up_sync(0xffffffffu, mincl, o);
      if (lane >= o) {
        incl += v;
        mincl += mv;
      }
    }
    const int excl = incl - sum, mexcl = mincl - msum;
    for (int s = beg; s < end; ++s) {
      tb.prefix[s] += excl;
      tb.mtp[s] += mexcl;
    }
    if (lane == 31) tb.prefix[nge] = incl;
  }
  __syncthreads();
  // from here on the kernel reads and writes global memory that the preceding
  // kernel may produce or consume: wait for it (programmatic dependent launch)
  griddep_wait();
  if (threadIdx.x == 0) MOE_TRACE_AT(1);
  // a pair's barriers are initialised before either CTA signals the other's
  if constexpr (CG == 2) cluster_sync();
  // the TMA producer (warp 0) issues no tcgen05 operation and does not read
  // the TMEM address, so it starts its loads without this fence
  if (warp != 0) tc_fence_after();
  if (threadIdx.x == 0) MOE_TRACE_AT(59);
  // The next kernel may start its own prologue now; it waits for this grid's
  // completion before touching memory.
  griddep_launch_dependents();
  if (threadIdx.x == 0) MOE_TRACE_AT(60);
  const uint32_t tmem_base = *tmem_slot;
  const int total = tb.prefix[nge];
  if (threadIdx.x == 0 && total >= 0) MOE_TRACE_AT(61);
  // Tile order: round-robin (unit, unit + nunits, ...), or, with many tiles per
  // unit, by ticket from a global counter: each unit's producer takes the next
  // tile when it starts one, so the units that hold long tiles (the weight
  // gradients of popular experts, K = their token count) take fewer, while
  // the tiles in flight stay neighbours (their A and B tiles shared in L2).
  // Tickets come in order, so a down tile of the fused forward only ever
  // waits for up tiles that running units hold.
  // (DYN: the kernel built with the ticket path; the round-robin build has
  // none of the queue code)
  const bool dyn = DYN && CG == 1 && P.sched != nullptr && total >= kDynMinTiles * nunits;
  // A consumer's next tile (-1: no more, -2: gave up waiting): round-robin
  // tiles are computed in place (`rr` starts at unit - nunits); ticket tiles
  // come from the queue, where `leader` releases the entry for the consumer
  // (one arrival per consumer).
  auto pop = [&](int& rr, int& qi, uint32_t& qph, bool leader) -> int {
    if (!dyn) {
      rr += nunits;
      return rr < total ? rr : -1;
    }
    if (!mbar_wait(&tq_full[qi], qph, &abort_flag, wait_ns)) return -2;
    const int v = tq[qi];
    __syncwarp(__activemask());
    if (leader) mbar_arrive(&tq_empty[qi]);
    if (++qi == kTileQ) {
      qi = 0;
      qph ^= 1;
    }
    return v;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int ti = 0, issued = 0;
      int qi = 0;
      uint32_t qph = 0;
      auto push = [&](int v) -> bool {  // publish the next tile to the consumers
        if (!mbar_wait(&tq_empty[qi], qph ^ 1, &abort_flag, wait_ns)) return false;
        tq[qi] = v;
        mbar_arrive(&tq_full[qi]);  // release: the index is visible with the phase
        if (++qi == kTileQ) {
          qi = 0;
          qph ^= 1;
        }
        return true;
      };
      int t = dyn ? atomicAdd(P.sched, 1) : unit;
      for (; t < total && ok; ++ti) {
        if (dyn && !push(t)) {
          ok = false;
          break;
        }
        // the next tile, taken now so that the ticket's round trip overlaps
        // this tile's loads
        const int t_next = dyn ? atomicAdd(P.sched, 1) : t + nunits;
        MOE_TRACE_TILE(ti, 0);
        const Tile tl = decode_tile<BMT>(tb, P, nge, t);
        const Problem& pr = P.pr[tl.p];
        const GroupedGemmDesc& g = pr.g;
        const int K = tb.K[tl.slot];
        const int nkb = (K + Elem<T>::BKE - 1) / Elem<T>::BKE;
        const int am = slot_base(g.a_m_base, tb, tl.slot) + tl.m0 + static_cast<int>(rank) * BM;
        const int ak = slot_base(g.a_k_base, tb, tl.slot);
        const int bn = slot_base(g.b_n_base, tb, tl.slot) + tl.n0 +
                       static_cast<int>(rank) * (pr.bn / CG);
        const int bk = slot_base(g.b_k_base, tb, tl.slot);
        // SwiGLU: gate columns n0.. then up columns N + n0.. of the expert
        const int up_shift = pr.epi == EPI_SWIGLU ? tb.N[tl.slot] - pr.bn / 2 : 0;
        if (g.dep_role == 2) {
          // rows of A written by problem 0 in this launch: wait for their row block
          const int s0 = tl.slot - P.pr[0].g.E;  // the same expert in problem 0
          const int blk = tb.mtp[s0] + tl.m0 / BMT;
          const int need = kEpiWarps * ((tb.N[s0] + P.pr[0].tile_n - 1) / P.pr[0].tile_n);
          if (blk >= g.dep_len) {
            if (g.status != nullptr) atomicExch(g.status, kStatusBadArg);
            abort_flag = 1;
            ok = false;
            break;
          }
          const uint64_t t0 = global_timer_ns();
          while (ld_acquire_gpu(g.dep + blk) < need) {
            if (abort_flag || global_timer_ns() - t0 > wait_ns) {
              abort_flag = 1;
              ok = false;
              break;
            }
          }
          if (!ok) break;
          fence_proxy_async_global();  // the TMA loads below see problem 0's stores
          MOE_TRACE_TILE(ti, 1);
          const int ntn = (tb.N[tl.slot] + pr.tile_n - 1) / pr.tile_n;
          if (atomicAdd(g.dep + g.dep_len + blk, 1) == ntn - 1) {  // last reader
            atomicExch(g.dep + blk, 0);
            atomicExch(g.dep + g.dep_len + blk, 0);
          }
        }
        if (ti == 0 && threadIdx.x == 0) MOE_TRACE_AT(62);
        if (tl.p == 0)
          ok = produce_tile<CFG0, T, CG>(ring, SB, S, full, empty, &abort_flag, wait_ns, &P.tmA[0],
                                         &P.tmB[0], nkb, am, ak, bn, bk, stage, phase, up_shift,
                                         issued);
        else
          ok = produce_tile<CFG1, T, CG>(ring, SB, S, full, empty, &abort_flag, wait_ns, &P.tmA[1],
                                         &P.tmB[1], nkb, am, ak, bn, bk, stage, phase, up_shift,
                                         issued);
        MOE_TRACE_TILE(ti, 2);
        t = t_next;
      }
      if (dyn && ok) ok = push(-1);  // no more tiles
      if (dyn) {
        // every unit ends with one ticket past the last tile (after an abort it
        // takes the rest first); the holder of the last ticket issued returns
        // the counter to zero for the next launch on this stream
        while (t < total) t = atomicAdd(P.sched, 1);
        if (t == total + nunits - 1) atomicExch(P.sched, 0);
      }
      if (!ok) drain_loads(full, S, stage, phase, issued, wait_ns);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int buf = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      int ti = 0, seen = 0;
      int qi = 0, rr = unit - nunits;
      uint32_t qph = 0;
      for (;; ++ti) {
        const int t = pop(rr, qi, qph, true);
        if (t < 0) break;
        const Tile tl = decode_tile<BMT>(tb, P, nge, t);
        const int K = tb.K[tl.slot];
        const int nkb = (K + Elem<T>::BKE - 1) / Elem<T>::BKE;
        bool free_acc;
        if constexpr (CG == 2) free_acc = mbar_wait_cluster(&acc_empty[buf], acc_phase ^ 1, &abort_flag, wait_ns);
        else free_acc = mbar_wait(&acc_empty[buf], acc_phase ^ 1, &abort_flag, wait_ns);
        if (!free_acc) break;
        tc_fence_after();
        MOE_TRACE_TILE(ti, 3);
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN_MAX);
        if (tl.p == 0)
          ok = mma_tile<CFG0, T, CG>(ring, SB, S, full, peer_full, empty, &abort_flag, wait_ns, d_tmem,
                                     K, nkb, stage, phase, seen);
        else
          ok = mma_tile<CFG1, T, CG>(ring, SB, S, full, peer_full, empty, &abort_flag, wait_ns, d_tmem,
                                     K, nkb, stage, phase, seen);
        if (!ok) break;
        MOE_TRACE_TILE(ti, 4);
        if constexpr (CG == 2) {
          if (nkb > 0) {
            tc_commit_pair(&acc_full[buf]);
          } else {
            mbar_arrive(&acc_full[buf]);
            mbar_arrive_remote(&acc_full[buf], 1);
          }
        } else {
          if (nkb > 0) tc_commit(&acc_full[buf]);
          else mbar_arrive(&acc_full[buf]);
        }
        buf ^= 1;
        if (buf == 0) acc_phase ^= 1;
      }
      // Make sure no MMA is still in flight before TMEM is released.
      tc_commit<CG>(drain);
      mbar_wait(drain, 0, &no_abort, wait_ns);
    } else if (CG == 2 && lane == 0) {
      // odd CTA of a pair: tell the even CTA's MMA issuer when each of this
      // CTA's stages has landed
      int stage = 0, seen = 0;
      uint32_t phase = 0;
      bool ok = true;
      int qi = 0, rr = unit - nunits;
      uint32_t qph = 0;
      while (ok) {
        const int t = pop(rr, qi, qph, true);
        if (t < 0) break;
        const Tile tl = decode_tile<BMT>(tb, P, nge, t);
        const int nkb = (tb.K[tl.slot] + Elem<T>::BKE - 1) / Elem<T>::BKE;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&full[stage], phase, &abort_flag, wait_ns)) {
            ok = false;
            break;
          }
          MOE_TRACE_KB(seen, 1);
          ++seen;
          mbar_arrive_remote(&peer_full[stage], 0);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // Each warp owns 32 accumulator rows (its TMEM lane quarter) and produces
    // them one slab at a time: 32 rows x 128 bytes (64 bf16 / 32 fp32 columns);
    // with 8 epilogue warps two warps share a quarter, each taking half of the
    // tile's slabs.
    // Every lane converts its own row into a shared staging slab laid out in
    // the TMA 128-byte swizzle (16-byte chunk c of row r at c ^ (r & 7)), then
    // one lane stores the slab with a TMA tensor store and the warp moves on;
    // two staging slabs per warp alternate (one slab in the ticket-order
    // build), so a slab is rewritten only after its previous store has
    // finished reading it.  Slabs that straddle an
    // expert's last row or column are stored by the lanes instead (row-major,
    // four 128-byte rows per instruction), never past the expert's extent.
    // The relu^2-derivative epilogue fetches its pre-activation slab by TMA
    // into the staging slab one slab ahead and computes in place.
    constexpr int EPC = Elem<T>::EPC;  // elements per 16-byte chunk
    constexpr int SLAB = 8 * EPC;      // columns per slab
    const int q = warp & 3;          // TMEM lane quarter (the hardware's warp % 4 rule)
    const int ew = warp - 2;         // epilogue warp index
    [[maybe_unused]] const int half = ew / 4;  // with 8 warps: which half of the column slabs
    uint8_t* stg_base = sEpi + ew * (kSlabs * 4096);
    uint64_t* ldb = epi_ld + ew * 2;
    uint32_t ld_phase = 0;  // bit i: parity of the next wait on ldb[i]
    uint32_t ld_pending = 0;  // bit i: a load into staging slab i not yet waited for
    int nbuf = 0;           // staging slab the next write goes to
    int buf = 0;
    uint32_t acc_phase = 0;
    const int rsub = lane >> 3;  // row within a 4-row group for the row-major phase
    const int csub = lane & 7;   // 16-byte chunk within a 128-byte row
    auto chunk_at = [&](uint8_t* stg, int row, int chunk) -> uint4* {
      return reinterpret_cast<uint4*>(stg + row * 128 + ((chunk ^ (row & 7)) << 4));
    };
    bool ok = true;
    int ti = 0;
    int qi = 0, rr = unit - nunits;
    uint32_t qph = 0;
    for (; ok; ++ti) {
      const int t = pop(rr, qi, qph, lane == 0);
      if (t < 0) break;
      const Tile tl = decode_tile<BMT>(tb, P, nge, t);
      const Problem& pr = P.pr[tl.p];
      const GroupedGemmDesc& g = pr.g;
      const int slot = tl.slot;
      const int M = tb.M[slot], N = tb.N[slot], K = tb.K[slot];
      const int epi = pr.epi;
      const bool dact = epi == EPI_DACT;
      const bool tma_out = pr.d_tma != 0;
      const CUtensorMap* tmD = &P.tmD[tl.p];
      const CUtensorMap* tmX = &P.tmX[tl.p];
      T* D = reinterpret_cast<T*>(g.d);
      T* AUX = reinterpret_cast<T*>(g.aux);
      T* AUX2 = reinterpret_cast<T*>(g.aux2);
      const int rbase = tl.m0 + static_cast<int>(rank) * BM + q * 32;  // this warp's first row
      const int rows_ok = min(32, M - rbase);  // may be <= 0
      const long long grow0 = static_cast<long long>(slot_base(g.d_m_base, tb, slot)) + rbase;
      const int gcol0 = slot_base(g.d_n_base, tb, slot) + tl.n0;
      const int ncols = min(pr.tile_n, N - tl.n0);
      // this warp's column slabs [s_lo, s_hi): all of them, or with two warps
      // per lane quarter the first or second half
      int s_lo = 0, s_hi = ncols;
      if constexpr (kEpiWarps == 8) {
        const int per = ((ncols + SLAB - 1) / SLAB + 1) / 2 * SLAB;
        s_lo = min(ncols, half * per);
        s_hi = min(ncols, s_lo + per);
      }
      // fetch an aux (pre-activation) slab into staging slab `b` (lane 0)
      auto fetch_aux = [&](int b, int s) {
        fence_proxy_async_smem();  // the lanes' reads of the slab precede the load
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_expect_tx(&ldb[b], 32 * 128);
          tma_load_2d(stg_base + b * 4096, tmX, &ldb[b], gcol0 + s, static_cast<int>(grow0));
        }
        ld_pending |= 1u << b;
      };
      if (dact) {
        // every earlier store has finished reading both staging slabs
        if (lane == 0) bulk_wait_group_read<0>();
        __syncwarp();
        nbuf = 0;
        if (rows_ok > 0 && s_lo < s_hi) fetch_aux(0, s_lo);  // overlaps the accumulator wait
      }
      if (!mbar_wait(&acc_full[buf], acc_phase, &abort_flag, wait_ns)) break;
      tc_fence_after();
      if (warp == 2 && lane == 0) MOE_TRACE_TILE(ti, 5);
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             static_cast<uint32_t>(buf * BN_MAX);
      // store the staged slab: TMA for full slabs, lanes for ragged ones
      auto put = [&](uint8_t* stg, const CUtensorMap* tm, T* dst, long long ld, int s,
                     int cvalid) {
        if (tma_out && cvalid == SLAB && rows_ok == 32) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(tm, stg, gcol0 + s, static_cast<int>(grow0));
            bulk_commit_group();
          }
        } else {
          __syncwarp();
          uint4 sv[8];
#pragma unroll
          for (int it = 0; it < 8; ++it) sv[it] = *chunk_at(stg, it * 4 + rsub, csub);
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int row = it * 4 + rsub;
            if (row < rows_ok && csub * EPC < cvalid)
              *reinterpret_cast<uint4*>(dst + (grow0 + row) * ld + gcol0 + s + csub * EPC) =
                  sv[it];
          }
          __syncwarp();
        }
      };
      // the next staging slab, once its previous TMA store has read it
      auto next_stage = [&]() -> uint8_t* {
        if (lane == 0) bulk_wait_group_read<kSlabs - 1>();
        __syncwarp();
        uint8_t* p = stg_base + nbuf * 4096;
        if constexpr (kSlabs == 2) nbuf ^= 1;
        return p;
      };
#pragma unroll 1
      for (int s = s_lo; s < s_hi && rows_ok > 0; s += SLAB) {
        const int cvalid = min(SLAB, ncols - s);
        if constexpr (((CFG0 | CFG1) & kCfgSwiglu) != 0) if (epi == EPI_SWIGLU) {
          // gate accumulator columns at tbase + s, up columns tile_n further
          const uint32_t tg = tbase + s, tu = tbase + pr.tile_n + s;
          auto stage_cols = [&](uint32_t tcol, T* dst, const CUtensorMap* tm, long long ld) {
            float v[SLAB];
            if (K > 0) {
              tmem_ld32(tcol, *reinterpret_cast<float(*)[32]>(&v[0]));
              if constexpr (SLAB > 32)
                if (cvalid > 32) tmem_ld32(tcol + 32, *reinterpret_cast<float(*)[32]>(&v[32]));
            } else {
#pragma unroll
              for (int i = 0; i < SLAB; ++i) v[i] = 0.f;
            }
            uint8_t* stg = next_stage();
#pragma unroll
            for (int j = 0; j < 8; ++j) *chunk_at(stg, lane, j) = pack_chunk<T>(&v[j * EPC]);
            put(stg, tm, dst, ld, s, cvalid);
          };
          if (AUX != nullptr) stage_cols(tg, AUX, tmX, g.ld_aux);     // gate
          if (AUX2 != nullptr) stage_cols(tu, AUX2, &P.tmY[tl.p], g.ld_aux2);  // up
          // out = silu(gate) * up from the fp32 accumulators, 32 columns at a time
          uint8_t* stg = next_stage();
#pragma unroll
          for (int h = 0; h < SLAB / 32; ++h) {
            float gv[32], uv[32], o[32];
            if (K > 0) {
              tmem_ld32(tg + 32 * h, gv);
              tmem_ld32(tu + 32 * h, uv);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) gv[i] = uv[i] = 0.f;
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = gv[i] / (1.0f + expf(-gv[i])) * uv[i];
#pragma unroll
            for (int j = 0; j < 32 / EPC; ++j)
              *chunk_at(stg, lane, h * (32 / EPC) + j) = pack_chunk<T>(&o[j * EPC]);
          }
          put(stg, tmD, D, g.ldd, s, cvalid);
          continue;
        }
        float v[SLAB];
        if (K > 0) {
          tmem_ld32(tbase + s, *reinterpret_cast<float(*)[32]>(&v[0]));
          if constexpr (SLAB > 32)
            if (cvalid > 32) tmem_ld32(tbase + s + 32, *reinterpret_cast<float(*)[32]>(&v[32]));
        } else {
#pragma unroll
          for (int i = 0; i < SLAB; ++i) v[i] = 0.f;
        }
        if (dact) {
          const int b = kSlabs == 2 ? ((s - s_lo) / SLAB) & 1 : 0;
          uint8_t* stg = stg_base + b * 4096;
          if (kSlabs == 1 && s != s_lo) {
            // one slab: this slab's pre-activation once the previous store has
            // read the slab
            if (lane == 0) bulk_wait_group_read<0>();
            __syncwarp();
            fetch_aux(0, s);
          }
          if (!mbar_wait(&ldb[b], (ld_phase >> b) & 1, &abort_flag, wait_ns)) {
            ok = false;
            break;
          }
          ld_phase ^= 1u << b;
          ld_pending &= ~(1u << b);
          if (kSlabs == 2 && s + SLAB < s_hi) {
            // prefetch the next aux slab into the other staging slab (its
            // previous store, if any, must have finished reading it)
            if (lane == 0) bulk_wait_group_read<0>();
            __syncwarp();
            fetch_aux(b ^ 1, s + SLAB);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float pr_[EPC], o[EPC];
            unpack_chunk<T>(*chunk_at(stg, lane, j), pr_);
#pragma unroll
            for (int i = 0; i < EPC; ++i) {
              const float gi = Cvt<T>::round(v[j * EPC + i]);
              o[i] = pr_[i] > 0.f ? gi * 2.0f * pr_[i] : 0.f;
            }
            *chunk_at(stg, lane, j) = pack_chunk<T>(o);
          }
          put(stg, tmD, D, g.ldd, s, cvalid);
          nbuf = kSlabs == 2 ? b ^ 1 : 0;  // the other slab is the older one now
        } else {
          if (epi == EPI_RELU2) {
#pragma unroll
            for (int i = 0; i < SLAB; ++i) v[i] = fmaxf(v[i], 0.f);
            if (AUX != nullptr) {
              uint8_t* stg = next_stage();
#pragma unroll
              for (int j = 0; j < 8; ++j) *chunk_at(stg, lane, j) = pack_chunk<T>(&v[j * EPC]);
              put(stg, tmX, AUX, g.ld_aux, s, cvalid);  // pre = relu(acc)
            }
#pragma unroll
            for (int i = 0; i < SLAB; ++i) v[i] = v[i] * v[i];
          }
          uint8_t* stg = next_stage();
#pragma unroll
          for (int j = 0; j < 8; ++j) *chunk_at(stg, lane, j) = pack_chunk<T>(&v[j * EPC]);
          put(stg, tmD, D, g.ldd, s, cvalid);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (warp == 2 && lane == 0) MOE_TRACE_TILE(ti, 6);
      if (lane == 0) {
        if (rank == 0) mbar_arrive(&acc_empty[buf]);
        else mbar_arrive_remote(&acc_empty[buf], 0);
      }
      if (g.dep_role == 1) {
        // this warp's stores of the tile are complete and visible before its
        // row block's count moves (the waiting problem loads them by TMA)
        if (lane == 0) bulk_wait_group_all();
        __syncwarp();
        __threadfence();
        if (lane == 0) {
          fence_proxy_async_global();
          const int blk = tb.mtp[slot] + tl.m0 / BMT;
          if (blk < g.dep_len) atomicAdd(g.dep + blk, 1);
        }
      }
      buf ^= 1;
      if (buf == 0) acc_phase ^= 1;
    }
    // after an abort: loads into the staging slabs must land before exit
    if (lane == 0)
      for (int b = 0; b < 2; ++b)
        if (ld_pending & (1u << b)) mbar_wait(&ldb[b], (ld_phase >> b) & 1, &no_abort, wait_ns);
    // stores must be complete (not only done reading smem) before exit
    if (lane == 0) bulk_wait_group_all();
    __syncwarp();
  }

  __syncthreads();
  if (threadIdx.x == 0) MOE_TRACE_AT(2);
  // neither CTA of a pair leaves (or frees TMEM) while the other may still
  // use its shared memory or tensor memory
  if constexpr (CG == 2) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<CG>(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && abort_flag) {
    for (int p = 0; p < P.nprob; ++p)
      if (P.pr[p].g.status != nullptr) atomicExch(P.pr[p].g.status, kStatusTimeout);
  }
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
// dtype: 0 bf16, 1 fp16, 2 fp32.
// mn_major: the tile feeds the MMA as an MN-major operand; fp32 ones then use
// the 128B swizzle with 32-byte granules that kind::tf32 reads MN-major.
int make_tmap(CUtensorMap* tm, const void* base, int dtype, long long inner, long long outer,
              long long ld, int box_inner, int box_outer, bool mn_major) {
  auto fn = encode_fn();
  if (!fn) return kStatusCuda;
  const int es = dtype == 2 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld * es) % 16 != 0) return kStatusBadArg;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * es)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = dtype == 2   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                              : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = fn(tm, dt,
                  2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  (dtype == 2 && mn_major) ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                           : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kStatusOk : kStatusBadArg;
}

template <typename T, int C0, int C1, int CG, bool DYN>
int launch_kernel(const MultiParams& P, int grid, cudaStream_t st) {
  auto kern = grouped_gemm_kernel<T, C0, C1, CG, DYN>;
  static bool attr_set[64] = {};   // per device
  static int max_pairs[64] = {};   // co-resident 2-CTA clusters, per device
  static std::mutex attr_mu;       // callers may be on several host threads
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return kStatusCuda;
  // Programmatic dependent launch: this grid's prologue (barrier init, TMEM
  // allocation, descriptor prefetch) overlaps the tail of the previous kernel.
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = CG;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = P.smem_bytes;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = CG == 2 ? 2 : 1;
  std::unique_lock<std::mutex> lock(attr_mu);
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax) !=
            cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) !=
            cudaSuccess)
      return kStatusCuda;
    if (CG == 2) {
      cfg.gridDim = dim3(2 * (num_sms() / 2));
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0)
        return kStatusCuda;
      max_pairs[dev] = n;
    }
    attr_set[dev] = true;
  }
  const int pairs = max_pairs[dev];
  lock.unlock();
  if (CG == 2) {
    grid = (grid / 2) * 2;
    if (grid > 2 * pairs || grid <= 0) grid = 2 * pairs;
  }
  cfg.gridDim = dim3(grid);
  if (cudaLaunchKernelEx(&cfg, kern, P) != cudaSuccess) return kStatusCuda;
  return cudaPeekAtLastError() == cudaSuccess ? kStatusOk : kStatusCuda;
}

// The ticket-order build when the host gave the launch a counter (single
// CTAs, many tiles expected), else the round-robin build.
template <typename T, int C0, int C1, int CG>
int launch(const MultiParams& P, int grid, cudaStream_t st) {
  if constexpr (CG == 1)
    if (P.sched != nullptr) return launch_kernel<T, C0, C1, CG, true>(P, grid, st);
  return launch_kernel<T, C0, C1, CG, false>(P, grid, st);
}

// One problem: any of the 8 operand configurations.
template <typename T, int CG>
int launch_single(int c, const MultiParams& P, int grid, cudaStream_t st) {
  switch (c) {
    case 0: return launch<T, 0, 0, CG>(P, grid, st);
    case 1: return launch<T, 1, 1, CG>(P, grid, st);
    case 2: return launch<T, 2, 2, CG>(P, grid, st);
    case 3: return launch<T, 3, 3, CG>(P, grid, st);
    case 4: return launch<T, 4, 4, CG>(P, grid, st);
    case 5: return launch<T, 5, 5, CG>(P, grid, st);
    case 6: return launch<T, 6, 6, CG>(P, grid, st);
    case 7: return launch<T, 7, 7, CG>(P, grid, st);
    // SwiGLU up projection (A K-major, B MN-major)
    case kCfgSwiglu | 2: return launch<T, kCfgSwiglu | 2, kCfgSwiglu | 2, CG>(P, grid, st);
    case kCfgSwiglu | 6: return launch<T, kCfgSwiglu | 6, kCfgSwiglu | 6, CG>(P, grid, st);
    default: return kStatusUnsupported;
  }
}
// Two problems: a K-major/K-major problem followed by an MN-major/MN-major one
// (the backward pairs), any N tiles.  Returns kStatusUnsupported otherwise.
template <typename T, int CG>
int launch_pair(int c0, int c1, const MultiParams& P, int grid, cudaStream_t st) {
  if ((c0 | c1) & kCfgSwiglu) return kStatusUnsupported;
  if ((c0 & 3) == 2 && (c1 & 3) == 2) {
    // A K-major, B MN-major twice: the fused up + down projection
    switch (((c0 >> 2) & 1) | (((c1 >> 2) & 1) << 1)) {
      case 0: return launch<T, 2, 2, CG>(P, grid, st);
      case 1: return launch<T, 6, 2, CG>(P, grid, st);
      case 2: return launch<T, 2, 6, CG>(P, grid, st);
      default: return launch<T, 6, 6, CG>(P, grid, st);
    }
  }
  if ((c0 & 3) != 0 || (c1 & 3) != 3) return kStatusUnsupported;
  const int k = ((c0 >> 2) & 1) | (((c1 >> 2) & 1) << 1);
  switch (k) {
    case 0: return launch<T, 0, 3, CG>(P, grid, st);
    case 1: return launch<T, 4, 3, CG>(P, grid, st);
    case 2: return launch<T, 0, 7, CG>(P, grid, st);
    default: return launch<T, 4, 7, CG>(P, grid, st);
  }
}

}  // namespace

static std::atomic<unsigned long long> g_wait_ns{MOE_WAIT_NS};

unsigned long long set_wait_ns(unsigned long long ns) {
  return g_wait_ns.exchange(ns == 0 ? MOE_WAIT_NS : ns);
}

int num_sms() {
  static std::atomic<int> cached{0};
  int n = cached.load(std::memory_order_relaxed);
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    cached.store(n, std::memory_order_relaxed);
  }
  return n;
}

// Ring stages and dynamic shared memory of a launch: the ring takes what the
// alignment pad, epilogue staging, barriers and the slot table leave.
static bool plan_smem(MultiParams& P, int bn_max, int cg) {
  const int nge = P.pr[0].g.E + (P.nprob > 1 ? P.pr[1].g.E : 0);
  P.stage_bytes = kABytes + bn_max / cg * 128;
  // the ticket-order build (a counter given, single CTAs) stages one slab per warp
  const bool dyn = cg == 1 && P.sched != nullptr;
  const int fixed = 1024 + epi_bytes(dyn) + kBarBytes + table_bytes(nge);
  int stages = (kSmemMax - fixed) / P.stage_bytes;
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2) return false;
  P.stages = stages;
  P.smem_bytes = fixed + stages * P.stage_bytes;
  return true;
}

template <typename T, int CG>
int dispatch(int used, int c0, int c1, const MultiParams& P, int grid, cudaStream_t st) {
  if (used == 1) return launch_single<T, CG>(c0, P, grid, st);
  return launch_pair<T, CG>(c0, c1, P, grid, st);
}

int dispatch_dtype(int dtype, int cg, int used, int c0, int c1, const MultiParams& P, int grid,
                   cudaStream_t st) {
  if (cg == 2) {
    if (dtype == 2) return dispatch<float, 2>(used, c0, c1, P, grid, st);
    if (dtype == 1) return dispatch<__half, 2>(used, c0, c1, P, grid, st);
    return dispatch<__nv_bfloat16, 2>(used, c0, c1, P, grid, st);
  }
  if (dtype == 2) return dispatch<float, 1>(used, c0, c1, P, grid, st);
  if (dtype == 1) return dispatch<__half, 1>(used, c0, c1, P, grid, st);
  return dispatch<__nv_bfloat16, 1>(used, c0, c1, P, grid, st);
}

// Tile-ticket counter of the launches on one (device, stream): zero between
// launches (each launch's last ticket holder returns it to zero), so launches
// that are ordered on one stream share it and launches on different streams
// never do.  Allocated (and zeroed on that stream) at the first launch outside
// stream capture; a stream that is capturing and has none yet gets null, and
// its launches take round-robin tiles.  A graph captured with a counter keeps
// it: its replays must not overlap launches on the capturing stream.
// (cudaStreamPerThread is one handle for all host threads: launches on it
// from several threads at once would share a counter.)
int* sched_counter(cudaStream_t st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  static std::mutex mu;
  static std::map<std::pair<int, uintptr_t>, int*> counters;
  const auto key = std::make_pair(dev, reinterpret_cast<uintptr_t>(st));
  std::lock_guard<std::mutex> lock(mu);
  const auto it = counters.find(key);
  if (it != counters.end()) return it->second;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return nullptr;
  }
  int* p = nullptr;
  if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (cudaMemsetAsync(p, 0, sizeof(int), st) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(p);
    return nullptr;
  }
  counters[key] = p;
  return p;
}

int run_grouped_gemms(const GemmOperands* ops, const GroupedGemmDesc* gs, const int* epis, int n,
                      int dtype, cudaStream_t st) {
  if (n <= 0 || n > kMaxProblems) return kStatusBadArg;
  MultiParams P;
  memset(&P, 0, sizeof(P));
  P.wait_ns = g_wait_ns.load(std::memory_order_relaxed);
  int bn_max = 128, grid = 0, used = 0;
  // CTA pairs (256-row tiles) only when every problem of the launch asks
  int cg = 2;
  for (int i = 0; i < n; ++i)
    if (gs[i].E != 0 && (ops[i].pair != 2 || epis[i] == EPI_SWIGLU || gs[i].dep_role != 0))
      cg = 1;
  // a dependent pair: problem 0 signals, problem 1 (same experts) waits
  if (n == 2 && (gs[0].dep_role != 0 || gs[1].dep_role != 0) &&
      (gs[0].dep_role != 1 || gs[1].dep_role != 2 || gs[0].E != gs[1].E || gs[0].E == 0 ||
       gs[0].dep == nullptr || gs[0].dep != gs[1].dep))
    return kStatusBadArg;
  for (int i = 0; i < n; ++i) {
    const GemmOperands& op = ops[i];
    const GroupedGemmDesc& g = gs[i];
    if (g.E == 0) continue;
    if (g.E < 0 || g.E > kMaxGroups) return kStatusUnsupported;
    if (op.a_rows <= 0 || op.a_cols <= 0 || op.b_rows <= 0 || op.b_cols <= 0)
      return kStatusBadArg;
    const int bn = op.bn == 256 ? 256 : 128;
    int s;
    // A is [a_rows, a_cols] row-major.  K-major A: rows are M, columns are K.
    // MN-major A: rows are K, columns are M.
    // boxes are one 128-byte swizzle row wide: 64 bf16 / 32 fp32 elements
    const int bke = dtype == 2 ? 32 : 64;
    if (op.a_mn) s = make_tmap(&P.tmA[used], op.a, dtype, op.a_cols, op.a_rows, op.lda, bke, bke, true);
    else s = make_tmap(&P.tmA[used], op.a, dtype, op.a_cols, op.a_rows, op.lda, bke, BM, false);
    if (s) return s;
    if (op.b_mn) s = make_tmap(&P.tmB[used], op.b, dtype, op.b_cols, op.b_rows, op.ldb, bke, bke, true);
    else s = make_tmap(&P.tmB[used], op.b, dtype, op.b_cols, op.b_rows, op.ldb, bke, bn / cg, false);
    if (s) return s;
    // epilogue maps: 32-row x 128-byte boxes in the staging-slab swizzle
    {
      const int sd = g.d_rows > 0
                         ? make_tmap(&P.tmD[used], g.d, dtype, g.ldd, g.d_rows, g.ldd, bke, 32, false)
                         : kStatusBadArg;
      int sx = kStatusOk;
      if (g.aux != nullptr && epis[i] != EPI_STORE)
        sx = g.aux_rows > 0 ? make_tmap(&P.tmX[used], g.aux, dtype, g.ld_aux, g.aux_rows,
                                        g.ld_aux, bke, 32, false)
                            : kStatusBadArg;
      if (epis[i] == EPI_DACT && sx != kStatusOk) return kStatusBadArg;
      int sy = kStatusOk;
      if (g.aux2 != nullptr && epis[i] == EPI_SWIGLU)
        sy = g.aux2_rows > 0 ? make_tmap(&P.tmY[used], g.aux2, dtype, g.ld_aux2, g.aux2_rows,
                                         g.ld_aux2, bke, 32, false)
                             : kStatusBadArg;
      P.pr[used].d_tma = (sd == kStatusOk && sx == kStatusOk && sy == kStatusOk) ? 1 : 0;
    }
    P.pr[used].g = g;
    P.pr[used].a_mn = op.a_mn;
    P.pr[used].b_mn = op.b_mn;
    P.pr[used].epi = epis[i];
    P.pr[used].bn = bn;
    P.pr[used].tile_n = epis[i] == EPI_SWIGLU ? bn / 2 : bn;
    if (epis[i] == EPI_SWIGLU && !op.b_mn) return kStatusUnsupported;  // gate/up boxes along N
    bn_max = bn > bn_max ? bn : bn_max;
    if (op.grid > grid) grid = op.grid;
    ++used;
  }
  if (used == 0) return kStatusOk;
  P.nprob = used;
  if (grid <= 0 || grid > num_sms()) grid = num_sms();
  // ticket-ordered tiles only where many tiles per CTA are expected (upper
  // estimate from the operands' extents; the kernel checks the real count)
  long long est = 0;
  for (int i = 0; i < n; ++i) {
    const GemmOperands& op = ops[i];
    const GroupedGemmDesc& g = gs[i];
    if (g.E <= 0) continue;
    const long long bn = op.bn == 256 ? 256 : 128;
    const long long m_ext = op.a_mn ? op.a_cols : op.a_rows;
    const long long n_ext = op.b_mn ? op.b_cols : op.b_rows;
    const long long m_blocks = (m_ext + BM - 1) / BM;
    const long long mb = g.m_src == DIM_CONST ? g.E * m_blocks : m_blocks;
    const long long n_per_expert = g.n_src == DIM_CONST ? n_ext : (n_ext + g.E - 1) / g.E;
    est += mb * ((n_per_expert + bn - 1) / bn);
  }
  P.sched = (cg == 1 && est >= static_cast<long long>(kDynMinTiles) * grid) ? sched_counter(st)
                                                                            : nullptr;
  if (!plan_smem(P, bn_max, cg)) return kStatusUnsupported;
#ifdef MOE_TRACE
  if (const char* g = getenv("MOE_TRACE_GRID")) grid = atoi(g);  // timeline experiments only
#endif
  const int c0 = cfg_of(P.pr[0].a_mn, P.pr[0].b_mn, P.pr[0].bn, P.pr[0].epi == EPI_SWIGLU);
  const int c1 = used > 1 ? cfg_of(P.pr[1].a_mn, P.pr[1].b_mn, P.pr[1].bn,
                                   P.pr[1].epi == EPI_SWIGLU)
                          : c0;
  int rc = dispatch_dtype(dtype, cg, used, c0, c1, P, grid, st);
  if (rc != kStatusUnsupported) return rc;
  if (P.pr[0].g.dep_role != 0) return kStatusUnsupported;  // dependent pairs launch together
  // no compiled pair for these configurations: one launch per problem
  for (int i = 0; i < used; ++i) {
    MultiParams Q = P;
    Q.nprob = 1;
    Q.tmA[0] = P.tmA[i];
    Q.tmB[0] = P.tmB[i];
    Q.tmD[0] = P.tmD[i];
    Q.tmX[0] = P.tmX[i];
    Q.tmY[0] = P.tmY[i];
    Q.pr[0] = P.pr[i];
    if (!plan_smem(Q, P.pr[i].bn, cg)) return kStatusUnsupported;
    const int ci = cfg_of(Q.pr[0].a_mn, Q.pr[0].b_mn, Q.pr[0].bn, Q.pr[0].epi == EPI_SWIGLU);
    rc = dispatch_dtype(dtype, cg, 1, ci, ci, Q, grid, st);
    if (rc != kStatusOk) return rc;
  }
  return kStatusOk;
}

int run_grouped_gemm(const GemmOperands& op, const GroupedGemmDesc& g, int epi, int dtype,
                     cudaStream_t st) {
  return run_grouped_gemms(&op, &g, &epi, 1, dtype, st);
}

}  // namespace moe

#ifdef MOE_TRACE
// Copy the per-CTA timeline of the last traced launch (two [160][64] uint64
// arrays of ns stamps, zero where no event was recorded) and clear it.
extern "C" __attribute__((visibility("default"))) int moe_trace_read(unsigned long long* host) {
  if (cudaMemcpyFromSymbol(host, moe::g_trace, sizeof(moe::g_trace)) != cudaSuccess) return -3;
  if (cudaMemcpyFromSymbol(host + moe::kTraceCtas * moe::kTraceSlots, moe::g_trace_kb,
                           sizeof(moe::g_trace_kb)) != cudaSuccess)
    return -3;
  static unsigned long long zeros[moe::kTraceCtas * moe::kTraceSlots] = {};
  if (cudaMemcpyToSymbol(moe::g_trace_kb, zeros, sizeof(zeros)) != cudaSuccess) return -3;
  return cudaMemcpyToSymbol(moe::g_trace, zeros, sizeof(zeros)) == cudaSuccess ? 0 : -3;
}
#endif
