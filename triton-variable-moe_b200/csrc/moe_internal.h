// Internal declarations shared by the .cu translation units of libmoe_b200.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace moe {

// Status codes (mirrored by the MOE_* constants of the public header).
constexpr int kStatusOk = 0;
constexpr int kStatusBadArg = -1;
constexpr int kStatusUnsupported = -2;
constexpr int kStatusCuda = -3;
constexpr int kStatusTimeout = -4;
constexpr int kStatusCapacity = -5;
constexpr int kStatusBadExpert = -6;

struct GroupedGemmDesc;

// Dense operand views of one grouped GEMM problem.  Both operands are
// row-major [rows, cols] with a row stride in elements.  `a_mn` / `b_mn`
// select the MN-major reading (rows are the reduction dimension).
struct GemmOperands {
  const void* a;
  long long a_rows, a_cols, lda;
  int a_mn;
  const void* b;
  long long b_rows, b_cols, ldb;
  int b_mn;
  int bn;    // N tile: 128 or 256
  int grid;  // CTAs; 0 = one per SM
  int pair;  // 2: 256-row tiles on 2-CTA clusters (cta_group::2); else 128-row tiles
};

int run_grouped_gemm(const GemmOperands& op, const GroupedGemmDesc& g, int epi, int dtype,
                     cudaStream_t st);
// Up to kMaxProblems independent grouped GEMMs in one persistent launch.
int run_grouped_gemms(const GemmOperands* ops, const GroupedGemmDesc* gs, const int* epis, int n,
                      int dtype, cudaStream_t st);  // dtype: 0 bf16, 1 fp16, 2 fp32 (tf32 MMA)

int num_sms();

// Limit (ns) of the grouped GEMM's device-side waits for launches that follow;
// 0 restores the default.  Returns the previous limit.
unsigned long long set_wait_ns(unsigned long long ns);

}  // namespace moe
