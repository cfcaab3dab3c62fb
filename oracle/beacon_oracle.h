/*
 * beacon_oracle.h -- CPU oracle for the beacon transformer hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA
 * kernels in beacon_b200/csrc: only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py may load it.  The product path
 * never calls into it and has no CPU fallback.
 *
 * Parity status: the reference (sienna-interwebs/beacon) has no numeric
 * implementation of any op (crates/beacon-ops/src/lib.rs:1 is empty and every
 * launch ends in LaunchError::Unimplemented, crates/beacon-cuda/src/runtime.rs:39-46),
 * so the op semantics below are a restatement of what the reference's launcher
 * signatures and adjoint-table entries imply.  The dtype codecs ARE pinned:
 * they restate crates/beacon-core/src/dtype.rs and are checked against that
 * file's known-answer tests (dtype.rs:224-265).  The attention / GEMM /
 * RMSNorm / SwiGLU results are "parity unpinned" by the reference; they are
 * cross-checked against an independent torch float64 restatement instead.
 *
 * Layouts are row-major and contiguous: matrices [rows, cols]
 * (crates/beacon-core/src/shape.rs:44-58), attention tensors [B, H, S, D]
 * (crates/beacon-macros/src/signature.rs:276), LSE [B, H, S] float32.
 * All dot products accumulate in double; results are stored as float32.
 */
#ifndef BEACON_ORACLE_H
#define BEACON_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- deterministic inputs -------------------------------------------------
 * Counter-based SplitMix64: value i of stream `seed` is the i-th output of a
 * SplitMix64 generator started at state `seed`.  Uniform u = top 24 bits / 2^24.
 * Normal: Box-Muller on the pair (u1 = (top24+1)/2^24, u2 = top24/2^24) of
 * outputs 2p and 2p+1, computed in double.  `offset` lets a caller generate
 * a slice [offset, offset+n) of the stream, so tensors can be filled in parts.
 */
uint64_t bo_splitmix64(uint64_t seed, uint64_t i);
void bo_fill_uniform(float* out, size_t n, float lo, float hi, uint64_t seed, uint64_t offset);
void bo_fill_normal(float* out, size_t n, float mean, float std, uint64_t seed, uint64_t offset);

/* ---- dtype codecs (crates/beacon-core/src/dtype.rs) ---------------------- */
uint16_t bo_bf16_from_f32(float x);        /* dtype.rs:58-66, RNE, NaN -> quiet  */
float bo_bf16_to_f32(uint16_t h);          /* dtype.rs:68-70                      */
uint8_t bo_fp8e4m3_from_f32(float x);      /* dtype.rs:163-195, saturate to 448   */
float bo_fp8e4m3_to_f32(uint8_t b);        /* dtype.rs:138-161                    */
void bo_f32_to_bf16(uint16_t* dst, const float* src, size_t n);
void bo_bf16_to_f32_n(float* dst, const uint16_t* src, size_t n);
void bo_round_bf16_inplace(float* x, size_t n);  /* x <- bf16(x) as float */
void bo_f32_to_fp8e4m3(uint8_t* dst, const float* src, size_t n);
void bo_fp8e4m3_to_f32_n(float* dst, const uint8_t* src, size_t n);

/* ---- GEMM family (crates/beacon-cuda/src/matmul.rs) ----------------------
 * matmul_fwd  (matmul.rs:18-29):  out[M,N] = lhs[M,K] . rhs[K,N]
 * matmul_bwd  (matmul.rs:31-44):  dlhs = dout . rhs^T ; drhs = lhs^T . dout
 * linear_fwd  (matmul.rs:46-58):  out = x . weight + bias   (weight [K,N], bias [N] or NULL)
 * linear_bwd  (matmul.rs:60-78):  dx = dy . W^T ; dW = x^T . dy ; db = sum_rows dy
 */
void bo_matmul_fwd(float* out, const float* lhs, const float* rhs, int64_t M, int64_t K, int64_t N);
void bo_matmul_bwd(float* dlhs, float* drhs, const float* dout, const float* lhs, const float* rhs,
                   int64_t M, int64_t K, int64_t N);
void bo_linear_fwd(float* out, const float* x, const float* w, const float* bias,
                   int64_t M, int64_t K, int64_t N);
void bo_linear_bwd(float* dx, float* dw, float* db, const float* dy, const float* x, const float* w,
                   int64_t M, int64_t K, int64_t N);

/* ---- causal scaled-dot-product attention (crates/beacon-cuda/src/attention.rs) ----
 * attention_fwd (attention.rs:21-40): O = softmax(scale Q K^T + mask) V and
 * LSE = natural-log logsumexp of each scaled, masked score row.
 * attention_bwd (attention.rs:42-64; adjoint entry crates/beacon-adjoint-table/src/lib.rs:86-99):
 * recomputes P from Q, K and LSE and returns dQ, dK, dV.
 * Q, O, dO, dQ: [B, Hq, S, D]; K, V, dK, dV: [B, Hkv, S, D]; query head h reads
 * KV head h / (Hq / Hkv).  Hq == Hkv is the reference's own signature.
 * Causal masking hides key j > query i.  scale <= 0 means 1/sqrt(D).
 */
void bo_attention_fwd(float* out, float* lse, const float* q, const float* k, const float* v,
                      int64_t B, int64_t Hq, int64_t Hkv, int64_t S, int64_t D, int causal, float scale);
void bo_attention_bwd(float* dq, float* dk, float* dv, const float* dout,
                      const float* q, const float* k, const float* v, const float* lse,
                      int64_t B, int64_t Hq, int64_t Hkv, int64_t S, int64_t D, int causal, float scale);
/* Run only the (b, h) query heads listed in `heads` (each index b*Hq+h); used for
 * sampled checks and the bounded CPU baseline at full sizes. */
void bo_attention_fwd_heads(float* out, float* lse, const float* q, const float* k, const float* v,
                            int64_t B, int64_t Hq, int64_t Hkv, int64_t S, int64_t D, int causal,
                            float scale, const int64_t* heads, int64_t nheads);
/* Forward of one query head for the listed query rows only, the rows spread over the
 * threads (a long head is checked on sampled rows in seconds).  q, k, v point at that
 * head's [S, D] rows; out [nrows, D], lse [nrows]. */
void bo_attention_fwd_rows(float* out, float* lse, const float* q, const float* k, const float* v,
                           int64_t S, int64_t D, int causal, float scale, const int64_t* rows, int64_t nrows);
/* Backward of one query head, its query rows spread over the threads (dk/dv summed from
 * per-thread double accumulators).  Same arithmetic as bo_attention_bwd for one head;
 * all pointers are that head's [S, D] / [S] rows. */
void bo_attention_bwd_head(float* dq, float* dk, float* dv, const float* dout, const float* q,
                           const float* k, const float* v, const float* lse, int64_t S, int64_t D, int causal,
                           float scale);

/* ---- RMSNorm (crates/beacon-cuda/src/norm.rs:19-51; adjoint lib.rs:70-77) ----
 * rms[t] = sqrt(mean_d x[t,d]^2 + eps); y = x * g / rms.  The saved statistic is rms.
 * bwd: dx = (g dy)/rms - x * sum_d(g dy x) / (dim rms^3); dg = sum_t dy x / rms.
 */
void bo_rmsnorm_fwd(float* y, float* rms, const float* x, const float* g, int64_t T, int64_t dim, float eps);
void bo_rmsnorm_bwd(float* dx, float* dg, const float* dy, const float* x, const float* rms,
                    const float* g, int64_t T, int64_t dim);

/* ---- LayerNorm (crates/beacon-cuda/src/norm.rs:55-95; adjoint lib.rs:78-85) ----
 * mean[t] = mean_d x[t,d]; invstd[t] = 1 / sqrt(mean_d (x[t,d] - mean[t])^2 + eps)
 * (biased variance); y = (x - mean) * invstd * g + b.  The saved statistics are mean, invstd.
 * bwd, with xh = (x - mean) invstd and e = g dy:
 *   dx = invstd * (e - mean_d e - xh * mean_d(e xh)); dg = sum_t dy xh; db = sum_t dy.
 * dg or db may be NULL.
 */
void bo_layernorm_fwd(float* y, float* mean, float* invstd, const float* x, const float* g, const float* b,
                      int64_t T, int64_t dim, float eps);
void bo_layernorm_bwd(float* dx, float* dg, float* db, const float* dy, const float* x, const float* mean,
                      const float* invstd, const float* g, int64_t T, int64_t dim);

/* ---- SwiGLU MLP (crates/beacon-cuda/src/mlp.rs:12-52; adjoint lib.rs:100-107) ----
 * out[T,dm] = (silu(x Wg) * (x Wu)) Wd, Wg/Wu [dm, F], Wd [F, dm], silu(z) = z / (1 + e^-z).
 * bwd recomputes gate and up and returns dx, dWg, dWu, dWd.
 */
void bo_swiglu_fwd(float* out, const float* x, const float* wg, const float* wu, const float* wd,
                   int64_t T, int64_t dm, int64_t F);
void bo_swiglu_bwd(float* dx, float* dwg, float* dwu, float* dwd, const float* dy, const float* x,
                   const float* wg, const float* wu, const float* wd, int64_t T, int64_t dm, int64_t F);

/* ---- residual add (crates/beacon-cuda/src/elementwise.rs:47-65; adjoint lib.rs:108-115) ---- */
void bo_residual_add_fwd(float* out, const float* a, const float* b, int64_t n);
void bo_residual_add_bwd(float* da, float* db, const float* dout, int64_t n);

/* Number of OpenMP threads the oracle uses (for reporting). */
int bo_num_threads(void);
void bo_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
