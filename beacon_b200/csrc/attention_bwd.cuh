// attention_bwd.cuh -- causal attention backward on tcgen05 tensor cores.
//
// Kernel ID `attention_adjoint_bwd` (crates/beacon-cuda/src/attention.rs:42-64); the
// adjoint entry (crates/beacon-adjoint-table/src/lib.rs:86-99) saves q, k, v, lse and
// recomputes the scores.  Three launches:
//   1. k_attn_bwd_prep   per query row: Dt = rowsum(dO * O), lse2 = lse * log2(e),
//                        zero the fp32 dQ accumulator.  (O is the forward output,
//                        recomputed by the forward kernel when the caller lacks it.)
//   2. k_attn_bwd_tc     one CTA per (128-key tile, KV head); loops over the query
//                        tiles (and, for grouped-query attention, the query heads of
//                        the group) that see those keys:
//        S^T  = K Q^T        (M=128 keys, N=128 queries, K=D)  -> TMEM [0,128)
//        dP^T = V dO^T       (same shape)                      -> TMEM [128,256)
//        softmax warps: P^T = exp2(S^T*scale*log2e - lse2), dS^T = P^T (dP^T - Dt);
//                       P^T (bf16) back into TMEM [0,64) as the A operand of dV,
//                       dS^T (bf16) into 128B-swizzled shared memory.
//        dV  += P^T dO       (A from TMEM, B = dO tile read MN-major)
//        dK  += dS^T Q       (A = dS^T K-major, B = Q tile read MN-major)
//        dQ_i = dS K         (A = the same dS^T tile read MN-major, B = K MN-major)
//                            -> TMEM [128, 128+D), added to the fp32 dQ accumulator
//                               with 16-byte vector atomics by four epilogue warps.
//      dK, dV accumulate in TMEM [256, 256+2D) and are written once at the end.
//   3. k_attn_dq_convert fp32 dQ accumulator -> output dtype.
#pragma once

#include "attention.cuh"
#include "sm100.cuh"

namespace beacon {

struct AttnBwdParams {
  int B, Hq, Hkv, S, S_pad;
  float scale;       // softmax scale (natural units)
  float scale_log2;  // scale * log2(e)
  int causal;
  const float* lse2;  // [B*Hq, S_pad]  lse * log2(e); +inf on padded rows
  const float* dt;    // [B*Hq, S_pad]  rowsum(dO * O); 0 on padded rows
  float* dq_acc;      // [B*Hq, S, D]   fp32, zeroed by the prep kernel
  __nv_bfloat16* dk;  // [B*Hkv, S, D]
  __nv_bfloat16* dv;  // [B*Hkv, S, D]
};

template <int D>
struct AttnBwdCfg {
  static constexpr uint32_t TILE_BYTES = 128 * D * 2;  // K, V, Q, dO tiles (128 rows x D)
  static constexpr uint32_t DS_BYTES = 128 * 128 * 2;
  static constexpr size_t SMEM_BYTES = 1024 + 6 * (size_t)TILE_BYTES + DS_BYTES + 512;
  static constexpr int THREADS = 320;  // producer, MMA, 4 softmax warps, 4 dQ warps
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t ST_COL = 0, DPT_COL = 128, DQ_COL = 128, DV_COL = 256, DK_COL = 256 + D;
};

enum : unsigned int {
  kSiteBwdKV = 0x301,
  kSiteBwdQDFull = 0x302,
  kSiteBwdQDEmpty = 0x303,
  kSiteBwdMmaDone = 0x304,
  kSiteBwdDqEmpty = 0x305,
  kSiteBwdStFull = 0x306,
  kSiteBwdDsFull = 0x307,
  kSiteBwdDqFull = 0x308,
  kSiteBwdDkvFull = 0x309,
  kSiteBwdDrain = 0x30a,
};

// ---------------------------------------------------------------------------
// 1. per-row preparation.  Half a warp per row for D=128 (16 lanes x 8 elements),
//    a quarter warp for D=64.  Grid-stride over B*Hq*S_pad rows.
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) k_attn_bwd_prep(const __nv_bfloat16* __restrict__ o,
                                                       const __nv_bfloat16* __restrict__ dout,
                                                       const float* __restrict__ lse, float* __restrict__ dt,
                                                       float* __restrict__ lse2, float* __restrict__ dq_acc,
                                                       long long n_bh, int S, int S_pad) {
  constexpr int LPR = D / 8;  // lanes per row
  constexpr int RPW = 32 / LPR;
  const long long total = n_bh * S_pad;
  const int lane = threadIdx.x & 31;
  const int sub = lane / LPR, l = lane % LPR;
  const long long warps = (long long)gridDim.x * (blockDim.x / 32);
  for (long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) / 32; w * RPW < total; w += warps) {
    const long long row = w * RPW + sub;
    float acc = 0.0f;
    bool valid = false;
    long long bh = 0;
    int q = 0;
    if (row < total) {
      bh = row / S_pad;
      q = (int)(row % S_pad);
      valid = q < S;
    }
    if (valid) {
      const long long base = (bh * S + q) * D + l * 8;
      const uint4 a = *reinterpret_cast<const uint4*>(o + base);
      const uint4 b = *reinterpret_cast<const uint4*>(dout + base);
      const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
      const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fa = __bfloat1622float2(pa[j]), fb = __bfloat1622float2(pb[j]);
        acc = fmaf(fa.x, fb.x, acc);
        acc = fmaf(fa.y, fb.y, acc);
      }
      float4* z = reinterpret_cast<float4*>(dq_acc + base);
      z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int off = LPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (row < total && l == 0) {
      dt[row] = valid ? acc : 0.0f;
      lse2[row] = valid ? lse[bh * S + q] * 1.4426950408889634f : INFINITY;
    }
  }
}

// fp32 accumulator -> bf16, 8 elements per thread per step
__global__ void k_attn_dq_convert(__nv_bfloat16* __restrict__ dq, const float* __restrict__ acc, long long n) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n / 8; i += stride) {
    const float4 a = reinterpret_cast<const float4*>(acc)[2 * i];
    const float4 b = reinterpret_cast<const float4*>(acc)[2 * i + 1];
    uint4 w;
    w.x = pack_bf16x2(a.x, a.y);
    w.y = pack_bf16x2(a.z, a.w);
    w.z = pack_bf16x2(b.x, b.y);
    w.w = pack_bf16x2(b.z, b.w);
    reinterpret_cast<uint4*>(dq)[i] = w;
  }
}

// ---------------------------------------------------------------------------
// 2. main backward kernel
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(320, 1)
    k_attn_bwd_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                  const AttnBwdParams p) {
  using Cfg = AttnBwdCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + Cfg::TILE_BYTES;
  uint8_t* sQ = sV + Cfg::TILE_BYTES;    // [2]
  uint8_t* sdO = sQ + 2 * Cfg::TILE_BYTES;  // [2]
  uint8_t* sdS = sdO + 2 * Cfg::TILE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sdS + Cfg::DS_BYTES);
  uint64_t* kv_full = bars + 0;
  uint64_t* qd_full = bars + 1;   // [2]
  uint64_t* qd_empty = bars + 3;  // [2]
  uint64_t* st_full = bars + 5;
  uint64_t* ds_full = bars + 6;
  uint64_t* dq_full = bars + 7;
  uint64_t* dq_empty = bars + 8;
  uint64_t* mma_done = bars + 9;
  uint64_t* dkv_full = bars + 10;
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id(), lane = lane_id();
  const int n_kvh = p.B * p.Hkv;
  const int jt = (int)(blockIdx.x / n_kvh);  // key tile: 0 first (the most causal work)
  const int kvz = (int)(blockIdx.x % n_kvh);
  const int b = kvz / p.Hkv, hk = kvz % p.Hkv;
  const int group = p.Hq / p.Hkv;
  const int j0 = jt * 128;
  const int n_q = (p.S + 127) / 128;
  const int it0 = p.causal ? jt : 0;
  const int iters_per_head = n_q - it0;
  const int n_iter = group * iters_per_head;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(st_full, 1);
    mbar_init(ds_full, 4);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 4);
    mbar_init(mma_done, 1);
    mbar_init(dkv_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmdO);
      mbar_arrive_expect_tx(kv_full, 2 * Cfg::TILE_BYTES);
      tma_load_rows<D>(sK, &tmK, kv_full, j0, kvz);
      tma_load_rows<D>(sV, &tmV, kv_full, j0, kvz);
      uint32_t issued = 0, par = 0;
      bool ok = true;
      for (int n = 0; n < n_iter && ok; ++n) {
        const int g = n / iters_per_head, it = it0 + n % iters_per_head;
        const int bh = b * p.Hq + hk * group + g;
        const int st = n & 1;
        const uint32_t ph = (n >> 1) & 1;
        if (!mbar_wait(&qd_empty[st], ph ^ 1u, abort_flag, kSiteBwdQDEmpty)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&qd_full[st], 2 * Cfg::TILE_BYTES);
        tma_load_rows<D>(sQ + st * Cfg::TILE_BYTES, &tmQ, &qd_full[st], it * 128, bh);
        tma_load_rows<D>(sdO + st * Cfg::TILE_BYTES, &tmdO, &qd_full[st], it * 128, bh);
        issued |= 1u << st;
        par = (par & ~(1u << st)) | (ph << st);
      }
      if (!ok) {
        volatile int no_abort = 0;
        mbar_wait(kv_full, 0, &no_abort, kSiteBwdDrain);
        for (int s = 0; s < 2; ++s)
          if (issued & (1u << s)) mbar_wait(&qd_full[s], (par >> s) & 1u, &no_abort, kSiteBwdDrain);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_f16(128, 128, false, false);  // S^T, dP^T
      constexpr uint32_t idesc_kv = make_idesc_f16(128, D, false, true);    // dV (A in TMEM), dK
      constexpr uint32_t idesc_q = make_idesc_f16(128, D, true, true);      // dQ
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV), ds_addr = smem_u32(sdS);
      bool ok = mbar_wait(kv_full, 0, abort_flag, kSiteBwdKV);
      for (int n = 0; n < n_iter && ok; ++n) {
        const int st = n & 1;
        const uint32_t ph = (n >> 1) & 1;
        if (!mbar_wait(&qd_full[st], ph, abort_flag, kSiteBwdQDFull)) { ok = false; break; }
        if (n > 0) {
          // previous dV/dK/dQ MMAs done (TMEM [0,64) P^T and the dS tile are free) and
          // the dQ epilogue has read TMEM [128, 128+D)
          if (!mbar_wait(mma_done, (n - 1) & 1, abort_flag, kSiteBwdMmaDone)) { ok = false; break; }
          if (!mbar_wait(dq_empty, (n - 1) & 1, abort_flag, kSiteBwdDqEmpty)) { ok = false; break; }
        }
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + st * Cfg::TILE_BYTES);
        const uint32_t do_addr = smem_u32(sdO + st * Cfg::TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_f16_ss(tmem + Cfg::ST_COL, make_sdesc_sw128(k_addr + off, 16, 1024),
                      make_sdesc_sw128(q_addr + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_f16_ss(tmem + Cfg::DPT_COL, make_sdesc_sw128(v_addr + off, 16, 1024),
                      make_sdesc_sw128(do_addr + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(st_full);
        if (!mbar_wait(ds_full, n & 1, abort_flag, kSiteBwdDsFull)) { ok = false; break; }
        tc_fence_after();
        const uint32_t acc_kv = (n > 0) ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // dV += P^T dO   (K = 128 queries)
          umma_f16_ts(tmem + Cfg::DV_COL, tmem + Cfg::ST_COL + kk * 8,
                      make_sdesc_sw128(do_addr + kk * 2048, 16384, 1024), idesc_kv, (acc_kv | kk) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // dK += dS^T Q
          umma_f16_ss(tmem + Cfg::DK_COL, make_sdesc_sw128(ds_addr + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                      make_sdesc_sw128(q_addr + kk * 2048, 16384, 1024), idesc_kv, (acc_kv | kk) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // dQ = dS K      (K = 128 keys)
          umma_f16_ss(tmem + Cfg::DQ_COL, make_sdesc_sw128(ds_addr + kk * 2048, 16384, 1024),
                      make_sdesc_sw128(k_addr + kk * 2048, 16384, 1024), idesc_q, kk > 0 ? 1u : 0u);
        umma_commit(&qd_empty[st]);
        umma_commit(dq_full);
        umma_commit(mma_done);
      }
      if (ok) umma_commit(dkv_full);
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, kSiteBwdDrain);
    }
  } else if (warp < 6) {
    // ---------------------------------------------------------------- softmax / dS (warps 2..5)
    const uint32_t quarter = warp & 3u;
    const int r = (int)(quarter * 32 + lane);  // key row within the tile == TMEM lane
    const int kj = j0 + r;
    const uint32_t lane_base = (quarter * 32u) << 16;
    bool ok = true;
    for (int n = 0; n < n_iter; ++n) {
      const int g = n / iters_per_head, it = it0 + n % iters_per_head;
      const int bh = b * p.Hq + hk * group + g;
      const int q0 = it * 128;
      if (!__all_sync(0xffffffffu, mbar_wait(st_full, n & 1, abort_flag, kSiteBwdStFull))) { ok = false; break; }
      tc_fence_after();
      const float* lse2p = p.lse2 + (long long)bh * p.S_pad + q0;
      const float* dtp = p.dt + (long long)bh * p.S_pad + q0;
      // keys beyond S, and (causal) queries before this key, get P = dS = 0
      const bool key_ok = kj < p.S;
      const int qmin = p.causal ? kj - q0 : -1;  // column index must be >= qmin
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t s[32], dp[32];
        tmem_ld32(tmem + lane_base + Cfg::ST_COL + c * 32, s);
        tmem_ld32(tmem + lane_base + Cfg::DPT_COL + c * 32, dp);
        tmem_wait_ld();
        float pv[32], dsv[32];
#pragma unroll
        for (int e4 = 0; e4 < 8; ++e4) {
          const float4 l4 = __ldg(reinterpret_cast<const float4*>(lse2p + c * 32 + e4 * 4));
          const float4 d4 = __ldg(reinterpret_cast<const float4*>(dtp + c * 32 + e4 * 4));
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
          const float dv[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int e = e4 * 4 + u;
            const int col = c * 32 + e;
            const bool live = key_ok && col >= qmin;
            const float pe = live ? ex2_approx(__uint_as_float(s[e]) * p.scale_log2 - lv[u]) : 0.0f;
            pv[e] = pe;
            dsv[e] = pe * (__uint_as_float(dp[e]) - dv[u]);
          }
        }
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) pk[e] = pack_bf16x2(pv[2 * e], pv[2 * e + 1]);
        // P^T chunk c (32 queries) -> TMEM columns [16c, 16c+16): over S^T columns already read
        tmem_st16(tmem + lane_base + Cfg::ST_COL + c * 16, pk);
        // dS^T chunk -> shared memory, K-major rows (key) of 64-query swizzled blocks
        uint8_t* blk = sdS + (c >> 1) * 16384;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          uint4 w;
          w.x = pack_bf16x2(dsv[8 * t + 0], dsv[8 * t + 1]);
          w.y = pack_bf16x2(dsv[8 * t + 2], dsv[8 * t + 3]);
          w.z = pack_bf16x2(dsv[8 * t + 4], dsv[8 * t + 5]);
          w.w = pack_bf16x2(dsv[8 * t + 6], dsv[8 * t + 7]);
          *reinterpret_cast<uint4*>(blk + sw128_offset((uint32_t)r, (uint32_t)((c & 1) * 4 + t))) = w;
        }
      }
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full);
    }
    // final dK, dV rows
    if (ok && __all_sync(0xffffffffu, mbar_wait(dkv_full, 0, abort_flag, kSiteBwdDkvFull))) {
      tc_fence_after();
      __nv_bfloat16* dvrow = p.dv + ((long long)kvz * p.S + kj) * D;
      __nv_bfloat16* dkrow = p.dk + ((long long)kvz * p.S + kj) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t a[32], k2[32];
        tmem_ld32(tmem + lane_base + Cfg::DV_COL + c * 32, a);
        tmem_ld32(tmem + lane_base + Cfg::DK_COL + c * 32, k2);
        tmem_wait_ld();
        if (kj < p.S) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 w, x;
            w.x = pack_bf16x2(__uint_as_float(a[e + 0]), __uint_as_float(a[e + 1]));
            w.y = pack_bf16x2(__uint_as_float(a[e + 2]), __uint_as_float(a[e + 3]));
            w.z = pack_bf16x2(__uint_as_float(a[e + 4]), __uint_as_float(a[e + 5]));
            w.w = pack_bf16x2(__uint_as_float(a[e + 6]), __uint_as_float(a[e + 7]));
            *reinterpret_cast<uint4*>(dvrow + c * 32 + e) = w;
            x.x = pack_bf16x2(__uint_as_float(k2[e + 0]) * p.scale, __uint_as_float(k2[e + 1]) * p.scale);
            x.y = pack_bf16x2(__uint_as_float(k2[e + 2]) * p.scale, __uint_as_float(k2[e + 3]) * p.scale);
            x.z = pack_bf16x2(__uint_as_float(k2[e + 4]) * p.scale, __uint_as_float(k2[e + 5]) * p.scale);
            x.w = pack_bf16x2(__uint_as_float(k2[e + 6]) * p.scale, __uint_as_float(k2[e + 7]) * p.scale);
            *reinterpret_cast<uint4*>(dkrow + c * 32 + e) = x;
          }
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- dQ epilogue (warps 6..9)
    const uint32_t quarter = warp & 3u;
    const int r = (int)(quarter * 32 + lane);  // query row within the tile == TMEM lane
    const uint32_t lane_base = (quarter * 32u) << 16;
    for (int n = 0; n < n_iter; ++n) {
      const int g = n / iters_per_head, it = it0 + n % iters_per_head;
      const int bh = b * p.Hq + hk * group + g;
      const int qi = it * 128 + r;
      if (!__all_sync(0xffffffffu, mbar_wait(dq_full, n & 1, abort_flag, kSiteBwdDqFull))) break;
      tc_fence_after();
      float* dst = p.dq_acc + ((long long)bh * p.S + qi) * D;
      // whole dQ row into registers, release TMEM to the next dP^T / dQ MMAs, then reduce
      uint32_t a[D];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) tmem_ld32(tmem + lane_base + Cfg::DQ_COL + c * 32,
                                                 *reinterpret_cast<uint32_t(*)[32]>(&a[c * 32]));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_empty);
      if (qi < p.S) {
#pragma unroll
        for (int e = 0; e < D; e += 4)
          red_add_v4(dst + e, __uint_as_float(a[e]) * p.scale, __uint_as_float(a[e + 1]) * p.scale,
                     __uint_as_float(a[e + 2]) * p.scale, __uint_as_float(a[e + 3]) * p.scale);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

}  // namespace beacon
