/*
 * beacon_cuda.h -- C ABI of libbeacon_cuda.so, the B200 (sm_100a) kernels behind
 * beacon's launcher traits.
 *
 * One entry point per kernel ID of crates/beacon-cuda (the IDs equal the
 * launcher strings of crates/beacon-adjoint-table/src/lib.rs:53-116).  Each takes
 * plain device pointers, explicit shapes, a dtype and a CUDA stream, because the
 * reference's typed traits drop the shapes before KernelLauncher::launch
 * (e.g. `let _ = (m, k, n)` at crates/beacon-cuda/src/matmul.rs:27).
 *
 * Conventions
 *  - Row-major contiguous tensors: matrices [rows, cols]; attention tensors
 *    [B, H, S, D]; LSE [B, H, S] float32; RMSNorm statistic rms and LayerNorm
 *    statistics mean, invstd: [tokens] float32.
 *  - `dtype` is a beacon_dtype (crates/beacon-core/src/dtype.rs:1-6 order).
 *    BEACON_BF16: bf16 operands, fp32 accumulation on tcgen05 tensor cores.
 *    BEACON_F32 : exact fp32 FFMA (no TF32) -- the 1e-5 parity path.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).  Every call is
 *    asynchronous on that stream and never synchronises the device, except
 *    where a comment says it may grow the library's internal workspace.
 *  - Concurrency: calls on different streams may overlap on the GPU, except that
 *    calls which take their scratch from the library's per-device workspace
 *    (workspace = NULL) share that one buffer: give each stream its own workspace
 *    when such calls may overlap.  The persistent kernels (attention forward, dK/dV, dQ)
 *    take their work items from one of 64 counter slots per device, rotating
 *    launch by launch and reset by each launch's last CTA: up to 64 such
 *    launches may be in flight on one device at once.
 *  - Return value: a beacon_status that maps 1:1 onto beacon-cuda's LaunchError
 *    variants (crates/beacon-cuda/src/error.rs:4-13); 0 is Ok.  The message of
 *    the last error on the calling thread is available from beacon_last_error().
 *  - No entry point falls back to the CPU.  A device without sm_100 support
 *    fails with BEACON_ERR_MODULE_LOAD.
 */
#ifndef BEACON_CUDA_H
#define BEACON_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* LaunchError variants, crates/beacon-cuda/src/error.rs:4-13 */
typedef enum beacon_status {
    BEACON_OK = 0,
    BEACON_ERR_UNIMPLEMENTED = 1,
    BEACON_ERR_INVALID_LAUNCH_CONFIG = 2,
    BEACON_ERR_MODULE_LOAD = 3,
    BEACON_ERR_FUNCTION_NOT_FOUND = 4,
    BEACON_ERR_CUDA = 5,
    BEACON_ERR_CUBLAS = 6,
    BEACON_ERR_OUT_OF_MEMORY = 7,
    BEACON_ERR_SHAPE_MISMATCH = 8
} beacon_status;

/* DType, crates/beacon-core/src/dtype.rs:1-7 */
typedef enum beacon_dtype {
    BEACON_F32 = 0,
    BEACON_F16 = 1,
    BEACON_BF16 = 2,
    BEACON_FP8E4M3 = 3
} beacon_dtype;

/* CastKind, crates/beacon-cuda/src/elementwise.rs:27-44 */
typedef enum beacon_cast_kind {
    BEACON_CAST_F32_TO_FP8E4M3 = 0,
    BEACON_CAST_FP8E4M3_TO_F32 = 1,
    BEACON_CAST_F32_TO_BF16 = 2,
    BEACON_CAST_BF16_TO_F32 = 3
} beacon_cast_kind;

/* ---- library / errors ----------------------------------------------------- */

/* Library ABI version (major * 10000 + minor * 100 + patch). */
int beacon_version(void);

/* Copies the calling thread's last error message into buf (NUL-terminated,
 * truncated to len) and returns the status that produced it. */
int beacon_last_error(char* buf, size_t len);

/* Reads and clears the device-side fault words of `device`:
 * out[0] fault code (0 none, 1 a bounded wait timed out), out[1] site,
 * out[2] number of faults since the last read.  Synchronises the device.
 * Replaces the kernel-completion check of crates/beacon-cuda/src/device.rs:72-74. */
int beacon_device_status(int device, unsigned int out[3]);

/* Number of kernels launched by this library since load (all devices, all threads). */
uint64_t beacon_launch_count(void);

/* Self-checks of device building blocks (no reference counterpart).
 * beacon_diag_wait_timeout: one warp on the current device waits on an mbarrier that
 * nothing completes, with the bounded wait every kernel uses but a limit of `limit_ns`
 * (at most 1 s); the wait gives up, records fault code 1 at site 0x501 (read it with
 * beacon_device_status), the bulk copy the kernel has in flight lands, its TMEM is freed
 * and it returns.  out: 3 device words = {gave up (1), first word of the copy (1),
 * TMEM released (1)}.
 * beacon_diag_exp2_poly: out[i] = 2^in[i] by the FMA-pipe polynomial the attention
 * softmax uses for part of its exponentials (n even); its stated bound is a relative
 * error below 7.5e-5 on [-125.5, 8] and an absolute error below 2^-125 beneath it. */
int beacon_diag_wait_timeout(uint64_t limit_ns, unsigned int* out, void* stream);
int beacon_diag_exp2_poly(float* out, const float* in, int64_t n, void* stream);

/* Device timing of the tensor-core kernels (k_gemm_bf16_tc, k_attn_fwd_tc,
 * k_attn_bwd_dkdv, k_attn_bwd_dq): while enabled, each launch is bracketed by CUDA events on its
 * own stream.  beacon_profile_read(name, ...) waits for those events and returns the
 * accumulated milliseconds and launch count for `name`; name == NULL resets.
 * No reference counterpart (the reference bench is a stub,
 * crates/beacon-bench/src/main.rs:1-3). */
void beacon_profile_enable(int on);
int beacon_profile_read(const char* kernel, double* total_ms, uint64_t* count);

/* ---- matmul / linear: crates/beacon-cuda/src/matmul.rs ---------------------- */

/* The tile shape the bf16 GEMM entry points choose for an [m, k] x [k, n] product with
 * 16-byte aligned rows on the current device: out[0] rows per tile (128, or 256 for an SM
 * pair), out[1] columns per tile, out[2] tiles, out[3] SMs per tile (1 or 2), out[4] the
 * device's SM count.  No counterpart in the reference: a planning query for launch
 * configuration and benchmarks (wave efficiency = tiles / (ceil(tiles / slots) x slots),
 * slots = SMs / SMs per tile). */
int beacon_matmul_plan(int64_t m, int64_t k, int64_t n, int32_t* out);

/* matmul_fwd (matmul.rs:18-29): out[m,n] = lhs[m,k] . rhs[k,n] */
int beacon_matmul_fwd(void* out, const void* lhs, const void* rhs, int64_t m, int64_t k, int64_t n,
                      int dtype, void* stream);

/* matmul_bwd (matmul.rs:31-44): dlhs[m,k] = dout . rhs^T ; drhs[k,n] = lhs^T . dout.
 * Either gradient pointer may be NULL to skip it. */
int beacon_matmul_bwd(void* dlhs, void* drhs, const void* dout, const void* lhs, const void* rhs,
                      int64_t m, int64_t k, int64_t n, int dtype, void* stream);

/* linear_fwd (matmul.rs:46-58): out[m,n] = x[m,k] . weight[k,n] + bias[n] (bias may be NULL). */
int beacon_linear_fwd(void* out, const void* x, const void* weight, const void* bias, int64_t m, int64_t k,
                      int64_t n, int dtype, void* stream);

/* fp8 e4m3 weights (DType::Fp8E4M3, crates/beacon-core/src/dtype.rs:6; codec dtype.rs:134-195;
 * the reference's "cublasLt fp8" / "fp32 master -> fp8 weights" plan, crates/beacon-cuda/Cargo.toml:7,
 * crates/beacon-train/Cargo.toml:7).  `dtype = BEACON_FP8E4M3` in beacon_matmul_fwd /
 * beacon_linear_fwd means: lhs / x, bias and out are bf16, rhs / weight is fp8 e4m3 [k, n]
 * with scale 1.  The _fp8w_ entry points take the per-tensor dequantisation scale:
 * out = (lhs . decode(rhs)) * scale (+ bias).  The weights are decoded to bf16 (exactly)
 * inside the GEMM pipeline -- TMA brings the fp8 bytes into shared memory, converter warps
 * decode them into the tensor core's operand layout -- so each weight byte is read from
 * HBM once; the scale is applied in the epilogue.  (lhs 16-byte aligned with k % 8 == 0,
 * weights 16-byte aligned with n % 16 == 0; other shapes decode to a bf16 copy in the
 * library workspace first.) */
int beacon_matmul_fp8w_fwd(void* out, const void* lhs, const void* rhs_fp8, float rhs_scale, int64_t m, int64_t k,
                           int64_t n, void* stream);
int beacon_linear_fp8w_fwd(void* out, const void* x, const void* weight_fp8, float weight_scale, const void* bias,
                           int64_t m, int64_t k, int64_t n, void* stream);
/* The same with the scale read from device memory (as beacon_quantize_fp8e4m3 writes it),
 * so no host round trip sits between quantising and using the weights; bias may be NULL. */
int beacon_linear_fp8w_fwd_devscale(void* out, const void* x, const void* weight_fp8, const float* weight_scale_dev,
                                    const void* bias, int64_t m, int64_t k, int64_t n, void* stream);

/* fp32 master -> fp8 e4m3 weights, one scale per tensor (the reference's "fp32 master ->
 * fp8 weights", crates/beacon-train/Cargo.toml:7; no scale convention is fixed there):
 *   amax = max |src| (NaN ignored), scale = amax / 448 (1 when amax is 0),
 *   out[i] = F8E4M3::from_f32(src[i] * (448 / amax))  (crates/beacon-core/src/dtype.rs:163-195,
 *   bit-exact, float32 arithmetic), so src ~ decode(out) * scale.
 * amax and scale are single floats in device memory (written on the stream). */
int beacon_quantize_fp8e4m3(void* out_fp8, float* scale, float* amax, const float* src, int64_t n, void* stream);

/* linear_bwd (matmul.rs:60-78): dx = dout . weight^T ; dweight = x^T . dout ; dbias = sum_rows dout.
 * Any gradient pointer may be NULL to skip it. */
int beacon_linear_bwd(void* dx, void* dweight, void* dbias, const void* dout, const void* x, const void* weight,
                      int64_t m, int64_t k, int64_t n, int dtype, void* stream);

/* ---- attention: crates/beacon-cuda/src/attention.rs ------------------------ */

/* attention_fwd (attention.rs:21-40), kernel `attention_adjoint_fwd`:
 * out = softmax(Q K^T / sqrt(head_dim) + causal mask) V, lse = natural-log logsumexp
 * per query row (float32).  q, k, v, out: [batch, heads, seqlen, head_dim]. */
int beacon_attention_adjoint_fwd(void* out, const void* q, const void* k, const void* v, float* lse,
                                 int64_t batch, int64_t heads, int64_t seqlen, int64_t head_dim, int causal,
                                 int dtype, void* stream);

/* attention_bwd (attention.rs:42-64), kernel `attention_adjoint_bwd`; adjoint entry
 * crates/beacon-adjoint-table/src/lib.rs:86-99 (saved q, k, v, lse; scores recomputed).
 * The forward output is not an argument: the forward kernel runs again, given the saved
 * lse, and forms rowsum(dO * O) from O in tensor memory (O is not written).  Scratch
 * (two fp32 values per query row): `workspace` of at least
 * beacon_attention_bwd_workspace_size(...) bytes, or NULL to use the library's
 * per-device workspace (grown with cudaMalloc on first use; the growth synchronises
 * the device). */
int beacon_attention_adjoint_bwd(void* dq, void* dk, void* dv, const void* dout, const void* q, const void* k,
                                 const void* v, const float* lse, int64_t batch, int64_t heads, int64_t seqlen,
                                 int64_t head_dim, int causal, int dtype, void* workspace,
                                 size_t workspace_bytes, void* stream);

size_t beacon_attention_bwd_workspace_size(int64_t batch, int64_t q_heads, int64_t seqlen, int64_t head_dim,
                                           int dtype);

/* Grouped-query variants.  No reference counterpart: attention.rs:28-31 has only
 * `heads`; these add kv_heads (q_heads % kv_heads == 0; query head h reads KV head
 * h / (q_heads / kv_heads)).  kv_heads == q_heads is exactly the entry points above.
 * k, v, dk, dv: [batch, kv_heads, seqlen, head_dim]. */
int beacon_attention_gqa_fwd(void* out, const void* q, const void* k, const void* v, float* lse, int64_t batch,
                             int64_t q_heads, int64_t kv_heads, int64_t seqlen, int64_t head_dim, int causal,
                             int dtype, void* stream);
int beacon_attention_gqa_bwd(void* dq, void* dk, void* dv, const void* dout, const void* q, const void* k,
                             const void* v, const float* lse, int64_t batch, int64_t q_heads, int64_t kv_heads,
                             int64_t seqlen, int64_t head_dim, int causal, int dtype, void* workspace,
                             size_t workspace_bytes, void* stream);

/* Backward that is also given the forward output `out`, so it skips the
 * recompute; for callers that keep O resident.  No reference counterpart. */
int beacon_attention_bwd_with_out(void* dq, void* dk, void* dv, const void* dout, const void* q, const void* k,
                                  const void* v, const void* out, const float* lse, int64_t batch,
                                  int64_t q_heads, int64_t kv_heads, int64_t seqlen, int64_t head_dim,
                                  int causal, int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* ---- RMSNorm: crates/beacon-cuda/src/norm.rs:19-51 -------------------------- */

/* rmsnorm_fwd (norm.rs:20-31): rms[t] = sqrt(mean(x[t]^2) + eps) (float32),
 * out = x * weight / rms.  The reference signature has no eps; its callers pass 1e-5. */
int beacon_rmsnorm_adjoint_fwd(void* out, const void* x, const void* weight, float* rms, int64_t tokens,
                               int64_t dim, float eps, int dtype, void* stream);

/* rmsnorm_bwd (norm.rs:33-50): dx = (w dy)/rms - x sum(w dy x)/(dim rms^3);
 * dweight = sum_t dy x / rms (NULL to skip).  Workspace as for attention. */
int beacon_rmsnorm_adjoint_bwd(void* dx, void* dweight, const void* dy, const void* x, const float* rms,
                               const void* weight, int64_t tokens, int64_t dim, int dtype, void* workspace,
                               size_t workspace_bytes, void* stream);

/* RMSNorm backward that allocates nothing.  No counterpart in the reference: it is
 * for callers that cannot allocate device memory themselves (a launcher that only
 * hands out pointers into one preallocated arena, a path that cannot afford the
 * first-call cudaMalloc and device synchronisation of the library's own workspace).
 * Same arithmetic as beacon_rmsnorm_adjoint_bwd (results agree up to the float32
 * summation order of dweight); the dweight partial sums live in a
 * fixed 4 MiB (1,048,576-float) array compiled into the library, which every GPU
 * that loads the library holds until exit.  dim above 1,048,576 is rejected with
 * BEACON_ERR_INVALID_LAUNCH_CONFIG.  The array's address is looked up on the first
 * call made on each device (make that call before any stream capture).  With CUDA's
 * lazy module loading (the default), the first call into this library on a device --
 * whichever entry point it is -- loads the library's module there, which places the
 * array and may synchronise; make one such call outside any latency-critical region,
 * or load eagerly with CUDA_MODULE_LOADING=EAGER.  All calls share the array: calls
 * that overlap on the GPU race and must be serialised. */
int beacon_rmsnorm_adjoint_bwd_noalloc(void* dx, void* dweight, const void* dy, const void* x, const float* rms,
                                       const void* weight, int64_t tokens, int64_t dim, int dtype, void* stream);

/* RMSNorm fused into the linear layer that consumes it: rmsnorm_fwd (norm.rs:20-31)
 * followed by linear_fwd (matmul.rs:46-58) as
 *     rmsnorm(x, g) . W + b = diag(1 / rms) . x . (diag(g) . W) + b.
 * beacon_rmsnorm_fold_weight writes w_out[i, j] = g[i] * w[i, j] (rounded to dtype), once
 * per weight version.  beacon_rmsnorm_linear_fwd then reads x once for its row statistic
 * rms[t] = sqrt(mean(x[t]^2) + eps) (written: the value rmsnorm_fwd saves for the
 * backward) and runs the GEMM on raw x and the folded weight with 1 / rms[t] applied to
 * each accumulator row in the epilogue (+ bias, may be NULL): no normalised copy of x is
 * written or read.  x [m, k], w_folded [k, n], out [m, n]; f32 or bf16.
 * No reference counterpart as one call (the reference has the two operators). */
int beacon_rmsnorm_fold_weight(void* w_out, const void* gain, const void* w, int64_t k, int64_t n, int dtype,
                               void* stream);
int beacon_rmsnorm_linear_fwd(void* out, float* rms, const void* x, const void* w_folded, const void* bias,
                              int64_t m, int64_t k, int64_t n, float eps, int dtype, void* stream);

/* ---- LayerNorm: crates/beacon-cuda/src/norm.rs:55-95 ----------------------- */

/* layernorm_fwd (norm.rs:56-73): mean[t] = mean_d x[t, d],
 * invstd[t] = 1 / sqrt(mean_d (x[t, d] - mean[t])^2 + eps) (biased variance; both float32),
 * out = (x - mean) * invstd * weight + bias.  The reference signature has no eps; 1e-5 is
 * the convention of the RMSNorm above.  The saved statistics are mean and invstd
 * (adjoint crates/beacon-adjoint-table/src/lib.rs:78-85). */
int beacon_layernorm_adjoint_fwd(void* out, const void* x, const void* weight, const void* bias, float* mean,
                                 float* invstd, int64_t tokens, int64_t dim, float eps, int dtype, void* stream);

/* layernorm_bwd (norm.rs:75-94): with xh = (x - mean) invstd and e = weight dy,
 * dx = invstd (e - mean_d e - xh mean_d(e xh)); dweight = sum_t dy xh; dbias = sum_t dy
 * (either may be NULL).  Workspace as for attention: 4 * min(tokens, 4 * SMs) * dim bytes
 * for each of dweight and dbias requested. */
int beacon_layernorm_adjoint_bwd(void* dx, void* dweight, void* dbias, const void* dy, const void* x,
                                 const float* mean, const float* invstd, const void* weight, int64_t tokens,
                                 int64_t dim, int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* ---- SwiGLU MLP: crates/beacon-cuda/src/mlp.rs:12-52 ----------------------- */

/* swiglu_fwd (mlp.rs:12-29): out[t, dm] = (silu(x Wg) * (x Wu)) Wd;
 * gate_proj, up_proj: [d_model, d_ff]; down_proj: [d_ff, d_model].
 * The gate and up GEMMs run as one tcgen05 GEMM with a SwiGLU epilogue. */
int beacon_swiglu_adjoint_fwd(void* out, const void* x, const void* gate_proj, const void* up_proj,
                              const void* down_proj, int64_t tokens, int64_t d_model, int64_t d_ff, int dtype,
                              void* workspace, size_t workspace_bytes, void* stream);

/* swiglu_bwd (mlp.rs:31-52); adjoint lib.rs:100-107 recomputes gate and up. */
int beacon_swiglu_adjoint_bwd(void* dx, void* dgate_proj, void* dup_proj, void* ddown_proj, const void* dy,
                              const void* x, const void* gate_proj, const void* up_proj, const void* down_proj,
                              int64_t tokens, int64_t d_model, int64_t d_ff, int dtype, void* workspace,
                              size_t workspace_bytes, void* stream);

size_t beacon_swiglu_workspace_size(int64_t tokens, int64_t d_model, int64_t d_ff, int dtype, int backward);

/* ---- pre-norm Llama-style block forward (no reference counterpart) ---------
 * The composition beacon-nn would make of rmsnorm_fwd (norm.rs:19-31), linear_fwd
 * (matmul.rs:46-58), attention_fwd (attention.rs:21-40), residual_add
 * (elementwise.rs:47-55) and swiglu_fwd (mlp.rs:12-29), in seven launches:
 *   h   = x + attention(rmsnorm(x, attn_norm) . w_qkv) . w_o        (causal)
 *   out = h + (silu(xn . w_gate) * (xn . w_up)) . w_down,  xn = rmsnorm(h, ffn_norm)
 * The QKV GEMM stores q, k, v head-major straight from its epilogue, attention writes
 * its output token-major, and both residual adds are GEMM epilogues.
 * x, out: [batch*seq, d_model]; attn_norm, ffn_norm: [d_model];
 * w_qkv: [d_model, (heads + 2*kv_heads)*head_dim] (query heads, then key heads, then
 * value heads); w_o: [heads*head_dim, d_model]; w_gate, w_up: [d_model, d_ff];
 * w_down: [d_ff, d_model].  bf16 only; head_dim 64 or 128; d_model and d_ff multiples
 * of 8; pointers 16-byte aligned.  Scratch (beacon_llama_block_workspace_size bytes,
 * or the library's workspace when `workspace` is NULL) holds, at the offsets the
 * layout in abi_block.inc gives, the normalised rows, both rms vectors, q, k, v, the
 * attention output, h and the SwiGLU activations. */
int beacon_llama_block_fwd(void* out, const void* x, const void* attn_norm, const void* w_qkv, const void* w_o,
                           const void* ffn_norm, const void* w_gate, const void* w_up, const void* w_down,
                           int64_t batch, int64_t seq, int64_t d_model, int64_t heads, int64_t kv_heads,
                           int64_t head_dim, int64_t d_ff, float eps, int dtype, void* workspace,
                           size_t workspace_bytes, void* stream);
size_t beacon_llama_block_workspace_size(int64_t batch, int64_t seq, int64_t d_model, int64_t heads,
                                         int64_t kv_heads, int64_t head_dim, int64_t d_ff, int dtype);

/* The same block with both RMSNorms folded into the GEMMs that consume them (six
 * launches and a 4-byte-per-row memset, no normalised activations written or read):
 * w_qkv_folded = diag(attn_norm) . w_qkv, w_gate_folded = diag(ffn_norm) . w_gate,
 * w_up_folded = diag(ffn_norm) . w_up, each made once per weight version with
 * beacon_rmsnorm_fold_weight.  The first norm's statistic is one read of x; the second's
 * is summed in the output projection's epilogue from the h it stores.  Same workspace. */
int beacon_llama_block_fwd_folded(void* out, const void* x, const void* w_qkv_folded, const void* w_o,
                                  const void* w_gate_folded, const void* w_up_folded, const void* w_down,
                                  int64_t batch, int64_t seq, int64_t d_model, int64_t heads, int64_t kv_heads,
                                  int64_t head_dim, int64_t d_ff, float eps, int dtype, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* ---- elementwise: crates/beacon-cuda/src/elementwise.rs -------------------- */

/* residual_add (elementwise.rs:47-55): out = a + b */
int beacon_residual_add_fwd(void* out, const void* a, const void* b, int64_t n, int dtype, void* stream);
/* residual_add_backward (elementwise.rs:57-65): d_a = d_b = d_out */
int beacon_residual_add_bwd(void* d_a, void* d_b, const void* d_out, int64_t n, int dtype, void* stream);
/* cast (elementwise.rs:120-128) with the reference's rounding rules (dtype.rs:58-66, 163-195). */
int beacon_cast(void* dst, const void* src, int64_t n, int kind, void* stream);

/* embedding_lookup (elementwise.rs:67-80): out[t, :] = table[indices[t], :], u32 indices.
 * embedding_backward (elementwise.rs:82-95): d_table[indices[t], :] += d_out[t, :] (atomic
 * adds; d_table is accumulated into, as its ReadWrite access in the reference's test says).
 * `vocab` (table rows) bounds the indices: an index >= vocab is not followed -- the forward
 * writes a zero row, the backward skips the token -- and the device fault word records code 3
 * (read it with beacon_device_status).  f32 or bf16 (bf16 adds round at every add). */
int beacon_embedding_lookup_fwd(void* out, const void* table, const uint32_t* indices, int64_t tokens, int64_t dim,
                                int64_t vocab, int dtype, void* stream);
int beacon_embedding_lookup_bwd(void* d_table, const void* d_out, const uint32_t* indices, int64_t tokens,
                                int64_t dim, int64_t vocab, int dtype, void* stream);

/* dropout_forward (elementwise.rs:97-108): element i is kept when u_i >= p, with
 * u_i = (splitmix64(seed, i) >> 40) / 2^24 (SplitMix64: z = seed + (i + 1) * 0x9E3779B97F4A7C15,
 * then the usual two xor-shift-multiply rounds), so the mask depends on (seed, i) only.
 * mask[i] = 1 / (1 - p) rounded to dtype for a kept element, 0 for a dropped one;
 * out = input * mask.  dropout_backward (elementwise.rs:110-118, no p): d_in = d_out * mask.
 * p >= 1 drops everything.  f32 or bf16; mask has the data type. */
int beacon_dropout_fwd(void* out, const void* input, void* mask, int64_t n, float p, uint64_t seed, int dtype,
                       void* stream);
int beacon_dropout_bwd(void* d_in, const void* d_out, const void* mask, int64_t n, int dtype, void* stream);

/* ---- arena launcher: the KernelLauncher::launch boundary ------------------
 * crates/beacon-cuda/src/runtime.rs:31-47 (Launcher::launch) and
 * crates/beacon-cuda/src/launcher.rs:21-63 (KernelArg = byte offset into one arena).
 * A Rust `Launcher` implements KernelLauncher::launch by forwarding here; the
 * typed traits' shapes, which they drop before launch, travel in `scalars`, in
 * this order per kernel ID (args in the typed trait's order):
 *   matmul_fwd/_bwd, linear_fwd/_bwd          m, k, n, dtype
 *   attention_adjoint_fwd/_bwd                batch, heads, seqlen, head_dim, causal, dtype[, kv_heads]
 *   rmsnorm_ / layernorm_adjoint_fwd/_bwd     tokens, dim, dtype[, eps as float32 bits]
 *   swiglu_adjoint_fwd/_bwd                   tokens, d_model, d_ff, dtype
 *   residual_add_fwd/_bwd                     n, dtype
 *   cast_*                                    n
 *   embedding_lookup_fwd/_bwd                 tokens, dim[, dtype]  (vocab = table extent / row)
 *   dropout_fwd                               n, p as float32 bits, seed[, dtype]
 *   dropout_bwd                               n[, dtype]                                   */
typedef struct beacon_arena beacon_arena;

typedef struct beacon_kernel_arg {
    uint64_t offset;     /* byte offset into the arena */
    uint64_t len_bytes;  /* extent, checked against the arena and the shapes */
    int32_t access;      /* 0 Read, 1 Write, 2 ReadWrite (launcher.rs:14-19) */
} beacon_kernel_arg;

/* Creates an arena of `bytes` device memory on `device` (256-byte aligned
 * regions are the caller's business, crates/beacon-core/src/arena.rs:7). */
beacon_arena* beacon_arena_create(int device, uint64_t bytes);
void beacon_arena_destroy(beacon_arena* arena);

/* The launcher's workspace (crates/beacon-cuda/src/runtime.rs:6-48 keeps one Launcher per
 * device; "kernels never allocate"): `bytes` of device memory owned by the arena, made once
 * at set-up (a second call replaces it, after a device synchronisation).  beacon_launch
 * hands it to every kernel ID that needs scratch (the attention, RMSNorm, LayerNorm and
 * SwiGLU backward, linear_bwd's dbias, the SwiGLU forward) and never allocates: when the
 * workspace is missing or too small the launch fails with BEACON_ERR_OUT_OF_MEMORY
 * ("requested / available").  Size it with the beacon_*_workspace_size functions. */
int beacon_workspace_create(beacon_arena* arena, uint64_t bytes);
void* beacon_arena_base(beacon_arena* arena);
uint64_t beacon_arena_size(beacon_arena* arena);

/* Dispatch by kernel ID string (the adjoint-table launcher names plus the
 * elementwise IDs).  `scalars` carries the dropped shapes, then dtype. */
int beacon_launch(beacon_arena* arena, const char* kernel, const beacon_kernel_arg* args, size_t nargs,
                  const int64_t* scalars, size_t nscalars, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* BEACON_CUDA_H */
