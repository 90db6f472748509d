// Persistent grouped GEMM on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// One launch computes every expert's tile of one of the six MoE GEMMs
// (up / down forward, dX / dW backward).  Per-expert problem geometry is not
// materialised as a sparse topology: each CTA derives it on device from the
// expert offset arrays (token offsets and weight offsets), builds a tile
// prefix table in shared memory and walks its share of the tiles.
//
// Roles inside a CTA (192 threads):
//   warp 0      TMA producer: streams A/B k-blocks into a ring of smem stages
//   warp 1      MMA issuer: one lane issues tcgen05.mma into a TMEM accumulator
//   warps 2..5  epilogue: tcgen05.ld the accumulator, fused activation, store
// The accumulator is double-buffered in TMEM so the epilogue of tile i
// overlaps the MMAs of tile i+1.
#pragma once
#include <cstdint>

namespace moe {

// Where a per-expert problem dimension comes from.
enum DimSrc : int {
  DIM_CONST = 0,   // a constant (the hidden size)
  DIM_TOKENS = 1,  // token rows of the expert: off[e+1] - off[e]
  DIM_WIDTH = 2,   // expert width: woff[e+1] - woff[e]
  DIM_HALF_WIDTH = 3,  // (woff[e+1] - woff[e]) / 2: SwiGLU, gate and up columns per expert
};
// Where a per-expert coordinate base comes from.
enum BaseSrc : int {
  BASE_ZERO = 0,
  BASE_TOK = 1,   // off[e]
  BASE_WOFF = 2,  // woff[e]
};
// Epilogue transforms.
enum EpiMode : int {
  EPI_STORE = 0,  // D = acc
  EPI_RELU2 = 1,  // aux = relu(acc); D = relu(acc)^2  (both rounded from fp32)
  EPI_DACT = 2,   // g = round(acc); D = pre > 0 ? g * 2 * pre : 0, pre read from aux
  EPI_SWIGLU = 3,  // the tile's B holds gate columns then up columns:
                   // D = silu(gate) * up; aux = gate, aux2 = up (both optional)
};

constexpr int kMaxGroups = 256;
constexpr int kMaxProblems = 2;  // independent problems per launch

struct GroupedGemmDesc {
  // expert metadata (device, int32)
  const int* tok_off;  // [E+1] row offsets of each expert in the padded token space
  const int* tok_cnt;  // [E] or null: caps the M extent of a token-row problem
  const int* w_off;    // [E+1] column offsets of each expert in the packed weights
  int E;
  int cdim;  // value of DIM_CONST
  int m_src, n_src, k_src;
  int a_m_base, a_k_base, b_n_base, b_k_base, d_m_base, d_n_base;
  // epilogue
  void* d;
  long long ldd;
  long long d_rows;  // rows of the D allocation (its tensor map extent)
  void* aux;
  long long ld_aux;
  long long aux_rows;  // rows of the aux allocation
  void* aux2;  // second epilogue output (SwiGLU: up), ld_aux2, aux2_rows rows
  long long ld_aux2;
  long long aux2_rows;
  int* status;  // device status word: set non-zero when a wait gave up
  // Row-block dependency between the two problems of one launch (dep_role 0:
  // none).  The signalling problem (1) is problem 0: each of its epilogue warps
  // adds 1 to dep[b] once its stores of a tile in row block b (expert e, rows
  // [m, m + 128)) have completed.  The waiting problem (2) is problem 1, over
  // the same experts and token rows: before loading a tile's A rows it waits
  // until dep[b] counts every epilogue warp of every problem-0 tile of that row
  // block.  dep[dep_len + b] counts the waiting tiles that passed; the last one
  // returns both words to zero, so the buffer is zero again after the launch.
  int* dep;
  int dep_len;
  int dep_role;
};

}  // namespace moe
