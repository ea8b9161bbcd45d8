// Host interface of the tcgen05 flash attention used by the OneTrans and
// LONGER backbones.
#pragma once

#include <cuda_runtime.h>

namespace mdl {

// Multi-head attention of a query SUFFIX over the keys of the same token
// sequence, with bottom-right causality and a per-sample valid-key start
// (reference MixedCausalAttention.attend_causal_suffix src/model.py:5617-5695
// over flash_attn_varlen_func):
//
//   qkv   [B, Lk, 3*D] bf16: per token Q | K | V, D = H * 32 (head h at h*32)
//   the queries are the last Lq tokens (rows Lk-Lq .. Lk-1) of each sample
//   key j is visible to query row p iff kstart[b] <= j and (!causal or j <= p or
//   j >= Lk - ktail or p >= Lk - ktail) and (j < Lk - kexcl or p >= Lk - kexcl)
//   out   [B, Lq, D] bf16, rows whose query has no visible key are zero
//   lse   [B, H, Lq] fp32: base-2 log-sum-exp of the scaled scores (+inf for
//         rows without a visible key), saved for the backward
//
// Backward: dqkv [B, Lk, 3*D] bf16 (every element written; Q rows that are not
// queries get zero), workspaces dq_acc fp32 [B, Lq, D] and dsum fp32 [B, H, Lq].
// Q of rows that are not queries is read (query tiles are 128 rows aligned to the
// end) but must only be finite: rows [max(0, Lk - 128*ceil(Lq/128)), Lk - Lq).
// head_dim is 32; H must be even for the forward (two heads per CTA).
struct FmhaArgs {
  const void* qkv = nullptr;
  void* out = nullptr;
  float* lse = nullptr;
  const int* kstart = nullptr;  // int32 [B]
  const void* dout = nullptr;   // bf16 [B, Lq, D]
  void* dqkv = nullptr;
  float* dq_acc = nullptr;
  float* dsum = nullptr;
  int B = 0, H = 0, Lk = 0, Lq = 0, hd = 32;
  bool causal = true;
  // With causal: the last ktail tokens (<= 128, all queries) see every key and are
  // seen by every query (LONGER's global tokens placed after the sequence).
  int ktail = 0;
  // With causal: the last kexcl (<= ktail) of those tokens are seen only by each
  // other (LONGER's candidate global tokens: no other token attends to them).
  int kexcl = 0;
  float scale = 0.f;            // softmax scale (1/sqrt(hd) when 0)
  int* err = nullptr;
};

cudaError_t fmha_fwd(const FmhaArgs& a, cudaStream_t stream);
cudaError_t fmha_bwd(const FmhaArgs& a, cudaStream_t stream);
// Which step of the last failing fmha_* call failed.
const char* fmha_last_error();

}  // namespace mdl
