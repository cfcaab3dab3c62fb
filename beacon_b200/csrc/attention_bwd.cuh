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
  static constexpr uint32_t STATS_BYTES = 2 * 128 * 4;  // lse2 and Dt of the current query tile
  static constexpr size_t SMEM_BYTES = 1024 + 6 * (size_t)TILE_BYTES + DS_BYTES + STATS_BYTES + 256;
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
  kSiteBwdStats = 0x30b,
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
//
// Each 128-query tile is processed as two halves of 64 queries so that the tensor
// core works on one half while the softmax warps turn the other into P^T / dS^T:
//   MMA issue order per tile:  S^T_0 dP^T_0  S^T_1 dP^T_1 | dV_0 dK_0 dQ_0 | dV_1 dK_1 dQ_1
//   softmax warps:                          (half 0)      (half 1)
// TMEM columns: S^T / P^T [0,128) (half h at 64h; P^T_h packed bf16 in its first 32
// columns), dP^T / dQ [128,256) (half h at 128+64h), dV [256,256+D), dK [256+D,256+2D).
// D=128: dQ^T_h = K^T dS^T_h (M = 128 head-dim lanes, N = 64 queries) so the dQ
//        epilogue thread of lane d adds dQ[q][d] for q = 0..63 with coalesced
//        128-byte fp32 reductions.
// D=64:  dQ = dS K once per tile after both halves (M = 128 queries, N = 64).
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(320, 1)
    k_attn_bwd_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                  const AttnBwdParams p) {
  using Cfg = AttnBwdCfg<D>;
  constexpr bool DQT = (D == 128);  // dQ^T per half (else dQ per tile)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + Cfg::TILE_BYTES;
  uint8_t* sQ = sV + Cfg::TILE_BYTES;       // [2]
  uint8_t* sdO = sQ + 2 * Cfg::TILE_BYTES;  // [2]
  uint8_t* sdS = sdO + 2 * Cfg::TILE_BYTES;
  float* sStats = reinterpret_cast<float*>(sdS + Cfg::DS_BYTES);  // [0,128) lse2, [128,256) Dt
  uint64_t* bars = reinterpret_cast<uint64_t*>(sdS + Cfg::DS_BYTES + Cfg::STATS_BYTES);
  uint64_t* kv_full = bars + 0;
  uint64_t* qd_full = bars + 1;    // [2] Q/dO stage
  uint64_t* qd_empty = bars + 3;   // [2]
  uint64_t* s_full = bars + 5;     // [2] half
  uint64_t* ds_full = bars + 7;    // [2] half
  uint64_t* dq_full = bars + 9;    // [2] half (D=64: [0] only)
  uint64_t* dq_empty = bars + 11;  // [2]
  uint64_t* half_done = bars + 13; // [2] every MMA reading P^T_h / dS^T_h has completed
  uint64_t* dkv_full = bars + 15;
  uint64_t* drain = bars + 16;
  uint64_t* stats_full = bars + 17;  // the 4 softmax warps stored this tile's lse2 / Dt
  uint64_t* stats_free = bars + 18;  // ... and finished reading them
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
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
      mbar_init(&s_full[i], 1);
      mbar_init(&ds_full[i], 4);
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_empty[i], 4);
      mbar_init(&half_done[i], 1);
    }
    mbar_init(dkv_full, 1);
    mbar_init(drain, 1);
    mbar_init(stats_full, 4);
    mbar_init(stats_free, 4);
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
      constexpr uint32_t idesc_s = make_idesc_f16(128, 64, false, false);   // S^T_h, dP^T_h
      constexpr uint32_t idesc_kv = make_idesc_f16(128, D, false, true);    // dV (A in TMEM), dK
      constexpr uint32_t idesc_qt = make_idesc_f16(128, 64, true, true);    // dQ^T_h (D = 128)
      constexpr uint32_t idesc_q = make_idesc_f16(128, D, true, true);      // dQ (D = 64)
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV), ds_addr = smem_u32(sdS);
      bool ok = mbar_wait(kv_full, 0, abort_flag, kSiteBwdKV);
      for (int n = 0; n < n_iter && ok; ++n) {
        const int st = n & 1;
        const uint32_t ph = (n >> 1) & 1;
        const uint32_t prev = (uint32_t)(n - 1) & 1u;
        if (!mbar_wait(&qd_full[st], ph, abort_flag, kSiteBwdQDFull)) { ok = false; break; }
        const uint32_t q_addr = smem_u32(sQ + st * Cfg::TILE_BYTES);
        const uint32_t do_addr = smem_u32(sdO + st * Cfg::TILE_BYTES);
        for (int h = 0; h < 2 && ok; ++h) {
          // S^T_h overwrites P^T_h of the previous tile, which the previous dV_h MMA reads:
          // tcgen05.mma executes in issue order, so that needs no wait.
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma_f16_ss(tmem + Cfg::ST_COL + 64 * h, make_sdesc_sw128(k_addr + off, 16, 1024),
                        make_sdesc_sw128(q_addr + off + h * 8192, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
          }
          // dP^T_h shares its columns with dQ, which the dQ warps read with tcgen05.ld:
          // those reads must have drained first.
          if (n > 0 && (DQT || h == 0) &&
              !mbar_wait(&dq_empty[DQT ? h : 0], prev, abort_flag, kSiteBwdDqEmpty)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma_f16_ss(tmem + Cfg::DPT_COL + 64 * h, make_sdesc_sw128(v_addr + off, 16, 1024),
                        make_sdesc_sw128(do_addr + off + h * 8192, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[h]);
        }
        if (!ok) break;
        for (int h = 0; h < 2; ++h) {
          if (!mbar_wait(&ds_full[h], (uint32_t)n & 1u, abort_flag, kSiteBwdDsFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t acc0 = (n > 0 || h > 0) ? 1u : 0u;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)  // dV += P^T_h dO_h   (K = 64 queries)
            umma_f16_ts(tmem + Cfg::DV_COL, tmem + Cfg::ST_COL + 64 * h + kk * 8,
                        make_sdesc_sw128(do_addr + h * 8192 + kk * 2048, 16384, 1024), idesc_kv, (acc0 | kk) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)  // dK += dS^T_h Q_h
            umma_f16_ss(tmem + Cfg::DK_COL, make_sdesc_sw128(ds_addr + h * 16384 + kk * 32, 16, 1024),
                        make_sdesc_sw128(q_addr + h * 8192 + kk * 2048, 16384, 1024), idesc_kv, (acc0 | kk) ? 1u : 0u);
          if constexpr (DQT) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)  // dQ^T_h = K^T dS^T_h   (K = 128 keys)
              umma_f16_ss(tmem + Cfg::DQ_COL + 64 * h, make_sdesc_sw128(k_addr + kk * 2048, 16384, 1024),
                          make_sdesc_sw128(ds_addr + h * 16384 + kk * 2048, 16384, 1024), idesc_qt,
                          kk > 0 ? 1u : 0u);
            umma_commit(&dq_full[h]);
          } else if (h == 1) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)  // dQ = dS K   (M = 128 queries, K = 128 keys)
              umma_f16_ss(tmem + Cfg::DQ_COL, make_sdesc_sw128(ds_addr + kk * 2048, 16384, 1024),
                          make_sdesc_sw128(k_addr + kk * 2048, 16384, 1024), idesc_q, kk > 0 ? 1u : 0u);
            umma_commit(&dq_full[0]);
          }
        }
        if (!ok) break;
        umma_commit(&qd_empty[st]);
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
    const bool key_ok = kj < p.S;
    const bool keys_full = j0 + 128 <= p.S;
    bool ok = true;
    for (int n = 0; n < n_iter && ok; ++n) {
      const int g = n / iters_per_head, it = it0 + n % iters_per_head;
      const int bh = b * p.Hq + hk * group + g;
      const int q0 = it * 128;
      // Stage this query tile's lse2 / Dt (1 KB) while the tensor core computes S^T and
      // dP^T: every softmax thread has finished the previous tile's reads (first barrier).
      const long long srow = (long long)bh * p.S_pad + q0 + r;
      const float l_r = __ldg(p.lse2 + srow), d_r = __ldg(p.dt + srow);
      if (n > 0 && !__all_sync(0xffffffffu, mbar_wait(stats_free, (uint32_t)(n - 1) & 1u, abort_flag, kSiteBwdStats))) {
        ok = false;
        break;
      }
      sStats[r] = l_r;
      sStats[128 + r] = d_r;
      __syncwarp();
      if (lane == 0) mbar_arrive(stats_full);
      if (!__all_sync(0xffffffffu, mbar_wait(stats_full, (uint32_t)n & 1u, abort_flag, kSiteBwdStats))) {
        ok = false;
        break;
      }
      // off-diagonal tiles need no mask: every key < S and every query >= every key
      const bool masked = !keys_full || (p.causal && it == jt);
      const int qmin = p.causal ? kj - q0 : -1;
      for (int h = 0; h < 2; ++h) {
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[h], (uint32_t)n & 1u, abort_flag, kSiteBwdStFull))) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t s[2][32], dp[2][32];
        tmem_ld32(tmem + lane_base + Cfg::ST_COL + 64 * h, s[0]);
        tmem_ld32(tmem + lane_base + Cfg::DPT_COL + 64 * h, dp[0]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 2; ++c) {  // 32 queries per chunk; chunk 1's TMEM load overlaps chunk 0
          if (c == 0) {
            tmem_ld32(tmem + lane_base + Cfg::ST_COL + 64 * h + 32, s[1]);
            tmem_ld32(tmem + lane_base + Cfg::DPT_COL + 64 * h + 32, dp[1]);
          }
          const int col0 = 64 * h + 32 * c;
          uint32_t pk[16];
          float dsv[32];
#pragma unroll
          for (int e4 = 0; e4 < 8; ++e4) {
            const float4 l4 = *reinterpret_cast<const float4*>(&sStats[col0 + 4 * e4]);
            const float4 d4 = *reinterpret_cast<const float4*>(&sStats[128 + col0 + 4 * e4]);
            const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
            const float dv[4] = {d4.x, d4.y, d4.z, d4.w};
            float pe[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int e = 4 * e4 + u;
              float pv = ex2_approx(fmaf(__uint_as_float(s[c][e]), p.scale_log2, -lv[u]));
              if (masked && !(key_ok && col0 + e >= qmin)) pv = 0.0f;
              pe[u] = pv;
              dsv[e] = pv * (__uint_as_float(dp[c][e]) - dv[u]);
            }
            pk[2 * e4] = pack_bf16x2(pe[0], pe[1]);
            pk[2 * e4 + 1] = pack_bf16x2(pe[2], pe[3]);
          }
          // P^T chunk -> TMEM columns [64h + 16c, +16): over S^T columns already read
          tmem_st16(tmem + lane_base + Cfg::ST_COL + 64 * h + 16 * c, pk);
          uint8_t* blk = sdS + h * 16384;
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            uint4 w;
            w.x = pack_bf16x2(dsv[8 * t + 0], dsv[8 * t + 1]);
            w.y = pack_bf16x2(dsv[8 * t + 2], dsv[8 * t + 3]);
            w.z = pack_bf16x2(dsv[8 * t + 4], dsv[8 * t + 5]);
            w.w = pack_bf16x2(dsv[8 * t + 6], dsv[8 * t + 7]);
            *reinterpret_cast<uint4*>(blk + sw128_offset((uint32_t)r, (uint32_t)(4 * c + t))) = w;
          }
          if (c == 0) tmem_wait_ld();
        }
        tmem_wait_st();
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&ds_full[h]);
          if (h == 1) mbar_arrive(stats_free);
        }
      }
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
    const uint32_t lane_base = (quarter * 32u) << 16;
    bool ok = true;
    for (int n = 0; n < n_iter && ok; ++n) {
      const int g = n / iters_per_head, it = it0 + n % iters_per_head;
      const int bh = b * p.Hq + hk * group + g;
      if constexpr (DQT) {
        const int d = (int)(quarter * 32 + lane);  // TMEM lane == head-dim index
        for (int h = 0; h < 2; ++h) {
          if (!__all_sync(0xffffffffu, mbar_wait(&dq_full[h], (uint32_t)n & 1u, abort_flag, kSiteBwdDqFull))) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t a[64];
          tmem_ld32(tmem + lane_base + Cfg::DQ_COL + 64 * h, *reinterpret_cast<uint32_t(*)[32]>(&a[0]));
          tmem_ld32(tmem + lane_base + Cfg::DQ_COL + 64 * h + 32, *reinterpret_cast<uint32_t(*)[32]>(&a[32]));
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&dq_empty[h]);
          const int qb = it * 128 + 64 * h;
          float* dst = p.dq_acc + ((long long)bh * p.S + qb) * D + d;
          const int nq = min(64, p.S - qb);
#pragma unroll
          for (int j = 0; j < 64; ++j)  // fully unrolled: a[] stays in registers
            if (j < nq) red_add_f32(dst + (long long)j * D, __uint_as_float(a[j]) * p.scale);
        }
      } else {
        const int qi = it * 128 + (int)(quarter * 32 + lane);  // TMEM lane == query row
        if (!__all_sync(0xffffffffu, mbar_wait(&dq_full[0], (uint32_t)n & 1u, abort_flag, kSiteBwdDqFull))) break;
        tc_fence_after();
        uint32_t a[D];
#pragma unroll
        for (int c = 0; c < D / 32; ++c)
          tmem_ld32(tmem + lane_base + Cfg::DQ_COL + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&a[c * 32]));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dq_empty[0]);
        if (qi < p.S) {
          float* dst = p.dq_acc + ((long long)bh * p.S + qi) * D;
#pragma unroll
          for (int e = 0; e < D; e += 4)
            red_add_v4(dst + e, __uint_as_float(a[e]) * p.scale, __uint_as_float(a[e + 1]) * p.scale,
                       __uint_as_float(a[e + 2]) * p.scale, __uint_as_float(a[e + 3]) * p.scale);
        }
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
