// Host interface of the tcgen05 batched GEMM.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mdl {

// Epilogue activation modes.
enum GemmAct : int {
  GEMM_ACT_NONE = 0,
  GEMM_ACT_GELU = 1,   // out = pre-activation, out2 = gelu(pre)
  GEMM_ACT_DGELU = 2,  // out = acc * gelu'(aux)
  GEMM_ACT_RELU = 3,   // out = relu(acc)
  GEMM_ACT_DRELU = 4,  // out = acc * (aux > 0)
  // GELU pair that saves the derivative instead of the pre-activation:
  GEMM_ACT_GELU_GRAD = 5,  // x = bf16(acc): out = gelu'(x), out2 = gelu(x)
  GEMM_ACT_DMUL = 6,       // out = acc * aux (aux = the saved derivative)
  GEMM_ACT_ADD = 7,        // out = acc + aux (a fused residual add)
};

// C[g] = epilogue(alpha * A[g] @ B[g]^T) for g in [0, G).
//   A[g] is M x K: K-major -> A[m,k] at A + g*gsA + m*lda + k
//                  MN-major -> A[m,k] at A + g*gsA + k*lda + m
//   B[g] is N x K: K-major -> B[n,k] at B + g*gsB + n*ldb + k
//                  MN-major -> B[n,k] at B + g*gsB + k*ldb + n
//   C[g] is M x N row-major: C[m,n] at out + g*gsC + m*ldc + n
// A batch stride of 0 with G > 1 shares that operand across the batch (one
// weight applied to every group). KG > 1 (with G == 1) sums KG products whose
// K ranges lie ksA / ksB elements apart: C = sum_j A_j @ B_j^T, each A_j, B_j
// of depth K (rows past K inside a range read as zeros), which is the weight
// gradient of a weight shared by rows that are not uniformly strided.
// A and B are bf16; C is bf16 or fp32. All leading dimensions and batch
// strides must be multiples of 8 elements (16 bytes) and the base pointers
// 16-byte aligned (TMA rule).
struct GemmArgs {
  const void* A = nullptr;
  long long lda = 0, gsA = 0;
  bool a_mn_major = false;
  const void* B = nullptr;
  long long ldb = 0, gsB = 0;
  bool b_mn_major = false;
  int M = 0, N = 0, K = 0, G = 1;
  int KG = 1;                       // K-range groups summed into one output
  long long ksA = 0, ksB = 0;       // element distance between K ranges
  // epilogue
  void* out = nullptr;
  long long ldc = 0, gsC = 0;
  bool out_fp32 = false;
  bool accumulate = false;          // out += result (fp32 or bf16 out)
  void* out2 = nullptr;             // bf16, same layout as out (GELU output)
  const float* bias = nullptr;      // bias[g*gs_bias + n]
  long long gs_bias = 0;
  const void* aux = nullptr;        // bf16 [.. ldc layout ..] for DGELU/DRELU
  long long ld_aux = 0, gs_aux = 0;
  float* colsum = nullptr;          // colsum[g*gs_colsum + n] += sum_m out[m,n]
  long long gs_colsum = 0;
  int act = GEMM_ACT_NONE;
  float alpha = 1.0f;
  int* err = nullptr;               // device error word
  int max_ctas = 0;                 // 0 = one CTA per SM
};

// Returns cudaSuccess or the launch/encode error.
cudaError_t gemm_bf16_tcgen05(const GemmArgs& args, cudaStream_t stream);

// CTA-pair (cta_group::2) tiles: -1 = by shape, 0 = off, 1 = wherever the shape allows.
// Returns the previous mode.
int gemm_pair_mode(int mode);

}  // namespace mdl
