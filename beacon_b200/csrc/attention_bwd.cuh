// attention_bwd.cuh -- causal attention backward on tcgen05 tensor cores, without atomics.
//
// Kernel ID `attention_adjoint_bwd` (crates/beacon-cuda/src/attention.rs:42-64); the
// adjoint entry (crates/beacon-adjoint-table/src/lib.rs:86-99) saves q, k, v, lse and
// recomputes the scores.  Three launches:
//   1. the row statistics Dt = rowsum(dO * O) and nlse2 = -lse * log2(e), padded to whole
//                       128-row tiles (-inf / 0), so no tile needs a row check; P =
//                       exp2(S * scale*log2e + nlse2) is one packed FMA and an exponential
//                       (MUFU; in dK/dV one pair in four of an unmasked tile runs as the
//                       FMA-pipe cubic exp2_poly2).  The
//                       drop-in entry, which has no O, runs the forward kernel's recompute
//                       form (k_attn_fwd_tc<D, true>: O stays in TMEM, its epilogue writes
//                       Dt and nlse2); given O, k_attn_bwd_prep reads it.
//   2. k_attn_bwd_dkdv  persistent, one CTA per SM over (128-key tile, KV head) items: dK
//                       and dV accumulate in TMEM over the query tiles (and grouped query
//                       heads) that see the keys.
//   3. k_attn_bwd_dq    persistent, one CTA per SM over (128-query tile, query head)
//                       items: dQ accumulates in TMEM over the key tiles the queries
//                       see, and is stored once in bf16.
// Each score tile is therefore computed twice.  The alternative -- one pass that adds
// every key tile's dQ contribution into an fp32 array in global memory -- moves 64 KB
// of fp32 reductions per tile through L2, which is both slower than the repeated S and
// dP products and a serialising step inside the pass.
//
// Both main kernels run 12 warps: warp 0 loads with TMA, warp 1 issues tcgen05.mma (the
// whole warp runs the issue loop, one elected lane issues), warps 2-3 idle, and warps
// 4-11 (two warpgroups, 2 warps per SM sub-partition) do the elementwise work; warps 0-3
// hand most of their registers to warps 4-11 (setmaxnreg: 128 x 120 + 256 x 192 = 384 x
// 168, the launch allocation; the MMA issuer keeps 120 registers so that no descriptor
// is spilled).
// Every MMA is M=128 x N=128 (N=64 MMAs take as long as N=128 ones on this tensor core).
#pragma once

#include "attention.cuh"
#include "sm100.cuh"

namespace beacon {

struct AttnBwdParams {
  int B, Hq, Hkv, S, S_pad;
  float scale;       // softmax scale (natural units)
  float scale_log2;  // scale * log2(e)
  int causal;
  const float* lse2;  // [B*Hq, S_pad]  -lse * log2(e); -inf on padded rows
  const float* dt;    // [B*Hq, S_pad]  rowsum(dO * O); 0 on padded rows
  __nv_bfloat16* dq;  // [B*Hq, S, D]
  __nv_bfloat16* dk;  // [B*Hkv, S, D]
  __nv_bfloat16* dv;  // [B*Hkv, S, D]
  int sched_slot;     // dQ kernel: its work counter (g_sched)
};

template <int D>
struct AttnBwdCfg {
  static constexpr uint32_t TILE_BYTES = 128 * D * 2;   // one 128-row tile of Q, K, V or dO
  static constexpr uint32_t STATS_BYTES = 2 * 128 * 4;  // lse2 and Dt of one query tile
  // dK/dV kernel: K, V, three stages of Q (with lse2), two of dO (with Dt), barriers and the
  // two-slot work-item ring.  The
  // 128-byte swizzled tiles need a 1024-byte aligned base; the window is allotted only 256
  // bytes of alignment slack (the whole 227 KB is in use), and the kernel reports
  // kFaultSmemAlign and does nothing if the window's placement needs more.
  static constexpr int DKDV_QST = 3;
  static constexpr uint32_t DKDV_BODY = (2 + DKDV_QST + 2) * TILE_BYTES + (DKDV_QST + 2) * 512 + 256;
  static constexpr uint32_t DKDV_SLACK = 256;
  static constexpr size_t DKDV_SMEM = (size_t)DKDV_BODY + DKDV_SLACK;
  // dQ kernel: Q, dO, three K stages, two V stages, barriers and the work-item ring.
  static constexpr size_t DQ_SMEM = 1024 + 7 * (size_t)TILE_BYTES + 512;
  static constexpr int THREADS = 384;
  static constexpr uint32_t TMEM_COLS = 512;
};

enum : unsigned int {
  kSiteBwdKV = 0x301,
  kSiteBwdQDFull = 0x302,
  kSiteBwdQDEmpty = 0x303,
  kSiteBwdStFull = 0x306,
  kSiteBwdDsFull = 0x307,
  kSiteBwdDkvFull = 0x309,
  kSiteBwdDrain = 0x30a,
  kSiteQKFull = 0x311,
  kSiteQKEmpty = 0x312,
  kSiteQVFull = 0x313,
  kSiteQVEmpty = 0x314,
  kSiteQSFull = 0x315,
  kSiteQDpFree = 0x316,
  kSiteQDsFull = 0x317,
  kSiteQDqFull = 0x318,
  kSiteQDrain = 0x319,
  kSiteQQd = 0x31a,
  kSiteQItem = 0x31b,
  kSiteBwdItem = 0x31c,
};

// ---------------------------------------------------------------------------
// 1. per-row preparation.  Half a warp per row for D=128 (16 lanes x 8 elements),
//    a quarter warp for D=64.  Grid-stride over B*Hq*S_pad rows.
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) k_attn_bwd_prep(const __nv_bfloat16* __restrict__ o,
                                                       const __nv_bfloat16* __restrict__ dout,
                                                       const float* __restrict__ lse, float* __restrict__ dt,
                                                       float* __restrict__ lse2, long long n_bh, int S, int S_pad) {
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
    }
#pragma unroll
    for (int off = LPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (row < total && l == 0) {
      dt[row] = valid ? acc : 0.0f;
      lse2[row] = valid ? lse[bh * S + q] * -1.4426950408889634f : -INFINITY;
    }
  }
}

// A score tile: D/16 K-steps of M=128 x N=128 with both operands K-major (A and B are
// 128 rows x D, each stored as D/64 swizzled 64-column blocks of 16 KB), from the tiles'
// K-major descriptors.  Called by the whole issuing warp; the elected `leader` lane
// executes the MMAs.
template <int D>
__device__ __forceinline__ void issue_score_tile(bool leader, uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc) {
  constexpr uint32_t idesc = make_idesc_f16(128, 128, false, false);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
    if (leader) umma_f16_ss(d_tmem, sdesc_adv(a_desc, off), sdesc_adv(b_desc, off), idesc, kk > 0 ? 1u : 0u);
  }
}
// K-major (score operands) and MN-major (row-major B of dV / dK / dQ / PV) descriptors of a
// 128-row x D tile at shared address `addr`.
__device__ __forceinline__ uint64_t tile_desc_k(uint32_t addr) { return make_sdesc_sw128(addr, 16, 1024); }
__device__ __forceinline__ uint64_t tile_desc_mn(uint32_t addr) { return make_sdesc_sw128(addr, 16384, 1024); }

// P^T for one warp's 64 query columns of a dK/dV tile: exp2(S^T * scale*log2e + lse2[q]),
// lse2 read from shared memory at `lse2_addr`.  MASKED zeroes the columns below
// `first_ok` (keys at or beyond S, or after the query); unmasked tiles take the variant
// without the selects.
template <bool MASKED>
__device__ __forceinline__ void bwd_p_cols(const uint32_t (&sv)[64], uint32_t lse2_addr, float scale_log2, int first_ok,
                                           float (&pe)[64]) {
#pragma unroll
  for (int e4 = 0; e4 < 16; ++e4) {
    const float4 l4 = lds_f4(lse2_addr + 16 * e4);
    float a0, a1, a2, a3;
    fma2(a0, a1, __uint_as_float(sv[4 * e4]), __uint_as_float(sv[4 * e4 + 1]), scale_log2, scale_log2, l4.x, l4.y);
    fma2(a2, a3, __uint_as_float(sv[4 * e4 + 2]), __uint_as_float(sv[4 * e4 + 3]), scale_log2, scale_log2, l4.z, l4.w);
    pe[4 * e4] = ex2_approx(a0);
    pe[4 * e4 + 1] = ex2_approx(a1);
    // one pair in four on the FMA pipe on unmasked tiles (dK/dV 0.6% faster at 256 heads, 2% at
    // 32; the dQ kernel measured 3% slower with the same split, so it keeps the exponential unit)
    if (!MASKED && (e4 & 1) == 0) {
      exp2_poly2(pe[4 * e4 + 2], pe[4 * e4 + 3], a2, a3);
    } else {
      pe[4 * e4 + 2] = ex2_approx(a2);
      pe[4 * e4 + 3] = ex2_approx(a3);
    }
    if (MASKED) {
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (4 * e4 + u < first_ok) pe[4 * e4 + u] = 0.0f;
    }
  }
}

// dS = P (dP - Dt) for one 32-key chunk of a dQ row, packed to bf16 pairs, with
// P = exp2(S * scale*log2e + nl2).  MASKED zeroes P from key `klim` on (keys at or beyond
// S, or after the query); unmasked tiles take the variant without the selects.
template <bool MASKED>
__device__ __forceinline__ void dq_ds_chunk(const uint32_t (&sc)[32], const uint32_t (&dpc)[32], float scale_log2,
                                            float nl2, float dtr, int klim, uint32_t (&pk)[16]) {
#pragma unroll
  for (int e = 0; e < 32; e += 2) {  // pairs: packed f32x2 arithmetic
    float a0, a1, t0, t1, d0, d1;
    fma2(a0, a1, __uint_as_float(sc[e]), __uint_as_float(sc[e + 1]), scale_log2, scale_log2, nl2, nl2);
    float p0 = ex2_approx(a0), p1 = ex2_approx(a1);
    if (MASKED) {
      if (e >= klim) p0 = 0.0f;
      if (e + 1 >= klim) p1 = 0.0f;
    }
    fma2(t0, t1, dtr, dtr, -1.0f, -1.0f, __uint_as_float(dpc[e]), __uint_as_float(dpc[e + 1]));
    mul2(d0, d1, p0, p1, t0, t1);
    pk[e >> 1] = pack_bf16x2(d0, d1);
  }
}

// ---------------------------------------------------------------------------
// 2. dK / dV.  Persistent: one CTA per SM walks work items (128-key tile, KV head), the first
//    its block index and the next ones from the launch's work counter, published by the
//    producer in a two-slot ring.  Query tiles are counted over all of the CTA's items (n),
//    so the Q / dO rings, the TMEM regions and the barrier phases run on across items: the
//    next item's K / V load once the current item's last S^T / dP^T have read K / V, its
//    first S^T / dP^T run behind the current item's last dK, and the warps write the
//    current item's dK / dV rows after the next item's first P and dS phases, while the
//    tensor core computes that item's second S^T; its first dV / dK MMAs wait for them.
//    Per query tile n of the item's 128 keys (M=128 keys x N=128 queries):
//     S^T(n)  = K Q(n)^T  -> TMEM region R_S(n)      dP^T(n) = V dO(n)^T -> region R_P(n)
//   The two 128-column regions X = [0,128) and Y = [128,256) swap roles every tile
//   (R_S(n) = X for even n, Y for odd n; R_P(n) is the other one), so the next tile's
//   S^T goes into the region whose dP^T the warps have just read, and its dP^T into the
//   region whose P^T / dS^T the dV / dK MMAs have just read.  MMA issue order per tile:
//     dV(n) += P^T(n) dO(n)   as soon as P^T(n) is stored
//     S^T(n+1) -> R_P(n)      as soon as every warp holds dP^T(n)
//     dK(n) += dS^T(n) Q(n)   as soon as dS^T(n) is stored
//     dP^T(n+1) -> R_S(n)     after dV(n) and dK(n) in issue order (MMAs run in order)
//   so the warps' dS phase (short) overlaps dV(n) and S^T(n+1), and their P phase (long:
//   the exponentials) overlaps dK(n-1) and dP^T(n): 32 MMAs of N=128 per tile.
//   Softmax warp (g, quarter): key rows 32*quarter.., queries 64g..64g+63; over the 64
//   S^T columns it has read it writes
//     P^T  = exp2(S^T * scale*log2e - lse2[q])   bf16 -> R_S(n) + [64g, 64g+32)
//     dS^T = P^T (dP^T - Dt[q])                  bf16 -> R_S(n) + [64g+32, 64g+64)
//   and dV / dK read them as the A operand from TMEM.
// TMEM: X [0,128) | Y [128,256) | dV [256,256+D) | dK [256+D,256+2D).
// ---------------------------------------------------------------------------
// Work items of the persistent dK/dV kernel: (128-key tile, KV head) in the grouped head
// order, key tile 0 (the most causal work) first.  The producer publishes them in a
// two-slot ring in shared memory (the kernel's shared memory has no room for more).
constexpr int kDkvItemRing = 2;
struct DkvItem {
  bool valid;
  int jt, kvz, b, hk;
  int it0, per_head, n_iter;  // first query tile, query tiles per query head, tiles of the item
};
__device__ __forceinline__ DkvItem dkv_item(const AttnBwdParams& p, int w) {
  DkvItem x;
  const int n_kvh = p.B * p.Hkv, n_kt = (p.S + 127) / 128;
  x.valid = w < n_kt * n_kvh;
  int jt = 0, kvz = 0;
  if (x.valid) grouped_order(w, n_kvh, n_kt, jt, kvz);
  x.jt = jt;
  x.kvz = kvz;
  x.b = kvz / p.Hkv;
  x.hk = kvz % p.Hkv;
  x.it0 = p.causal ? jt : 0;
  x.per_head = n_kt - x.it0;
  x.n_iter = x.valid ? (p.Hq / p.Hkv) * x.per_head : 0;
  return x;
}

template <int D>
__global__ void __launch_bounds__(384, 1)
    k_attn_bwd_dkdv(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                    const AttnBwdParams p) {
  using Cfg = AttnBwdCfg<D>;
  constexpr uint32_t TILE = Cfg::TILE_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  if ((uint32_t)(smem - smem_raw) > Cfg::DKDV_SLACK) {  // uniform over the grid: nothing has started
    if (threadIdx.x == 0) {
      record_fault(kFaultSmemAlign, kSiteBwdKV);
      sched_finish(p.sched_slot);
    }
    return;
  }
  uint8_t* sK = smem;
  uint8_t* sV = sK + TILE;
  constexpr int QST = Cfg::DKDV_QST;
  uint8_t* sQ = sV + TILE;         // [QST]
  uint8_t* sdO = sQ + QST * TILE;  // [2]
  float* sLse = reinterpret_cast<float*>(sdO + 2 * TILE);  // [QST][128] lse2, with Q
  float* sDt = sLse + QST * 128;                            // [2][128] Dt, with dO
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDt + 2 * 128);
  constexpr int NB = D / 64;        // 64-column blocks of a tile
  uint64_t* kv_full = bars + 0;     // an item's K and V
  // [3][2] per Q stage and column block (the last block's barrier also carries lse2): the
  // score MMAs of block 0 start while block 1 is still landing
  uint64_t* q_full = bars + 1;
  uint64_t* q_empty = bars + 7;    // [3] Q read by S^T and dK
  uint64_t* do_full = bars + 10;   // [2] dO and Dt of a query tile
  uint64_t* do_empty = bars + 12;  // [2] dO read by dP^T and dV
  uint64_t* s_full = bars + 14;    // S^T(n) computed
  uint64_t* dp_full = bars + 15;   // dP^T(n) computed
  uint64_t* p_ready = bars + 16;   // P^T(n) stored by all 8 warps
  uint64_t* rp_free = bars + 17;   // dP^T(n) read by all 8 warps: R_P(n) may take S^T(n+1)
  uint64_t* ds_ready = bars + 18;  // dS^T(n) stored by all 8 warps
  uint64_t* dkv_full = bars + 19;  // an item's dK, dV complete in TMEM
  uint64_t* drain = bars + 20;
  uint64_t* kv_empty = bars + 21;  // an item's last S^T and dP^T have read K and V
  uint64_t* item_full = bars + 22;                  // [2] item published by the producer
  uint64_t* item_empty = item_full + kDkvItemRing;  // [2] read by the MMA warp and the 8 softmax warps
  uint64_t* acc_free = item_empty + kDkvItemRing;   // an item's dV, dK read out of TMEM by the 8 warps
  int* s_item = reinterpret_cast<int*>(acc_free + 1);  // [2] item indices
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_item + kDkvItemRing);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  constexpr uint32_t T_DV = 256, T_DK = 256 + D;

  const uint32_t warp = warp_id(), lane = lane_id();
  const int group = p.Hq / p.Hkv;
  const int n_items = ((p.S + 127) / 128) * p.B * p.Hkv;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int i = 0; i < QST; ++i) {
      mbar_init(&q_full[2 * i], 1);
      mbar_init(&q_full[2 * i + 1], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&do_full[i], 1);
      mbar_init(&do_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(p_ready, 8);
    mbar_init(rp_free, 8);
    mbar_init(ds_ready, 8);
    mbar_init(dkv_full, 1);
    mbar_init(drain, 1);
    for (int i = 0; i < kDkvItemRing; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 9);
    }
    mbar_init(acc_free, 8);
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

  // The ci-th item of this CTA from the ring (every role but the producer); `valid` false at
  // the end of the CTA's work or when the wait gave up (then `ok` is cleared).
  auto read_item = [&](int ci, bool& ok) -> DkvItem {
    const int slot = ci % kDkvItemRing;
    if (!mbar_wait(&item_full[slot], (uint32_t)(ci / kDkvItemRing) & 1u, abort_flag, kSiteBwdItem)) {
      ok = false;
      return dkv_item(p, INT32_MAX);
    }
    return dkv_item(p, s_item[slot]);
  };

  if (warp < 4) {
    warpgroup_reg_dealloc<120>();
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------------------- producer
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmdO);
      // per item: K and V (once the previous item's last S^T and dP^T have read them), then
      // Q (with lse2) and dO (with Dt) of its query tiles into rings that run on across
      // items, Q three deep: Q(n+3) loads once dK(n) has read Q(n), a whole tile before
      // S^T(n+3) needs it.  n counts query tiles over all of the CTA's items.
      uint32_t n = 0, kviss = 0, kvpar = 0, qiss = 0, qpar = 0, diss = 0, dpar = 0;
      bool ok = true;
      for (int ci = 0; ok; ++ci) {
        // fetch the CTA's next item and publish it (an index >= n_items ends every role)
        const int w = ci == 0 ? (int)blockIdx.x : sched_fetch(p.sched_slot);
        const int slot = ci % kDkvItemRing;
        if (!mbar_wait(&item_empty[slot], ((uint32_t)(ci / kDkvItemRing) & 1u) ^ 1u, abort_flag, kSiteBwdItem)) {
          ok = false;
          break;
        }
        s_item[slot] = w < n_items ? w : n_items;
        mbar_arrive(&item_full[slot]);
        const DkvItem x = dkv_item(p, w);
        if (!x.valid) break;
        if (!mbar_wait(kv_empty, ((uint32_t)ci & 1u) ^ 1u, abort_flag, kSiteBwdKV)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(kv_full, 2 * TILE);
        tma_load_rows<D>(sK, &tmK, kv_full, x.jt * 128, x.kvz);
        tma_load_rows<D>(sV, &tmV, kv_full, x.jt * 128, x.kvz);
        kviss = 1;
        kvpar = (uint32_t)ci & 1u;
        for (int m = 0; m < x.n_iter; ++m, ++n) {
          const int g = m / x.per_head, it = x.it0 + m % x.per_head;
          const int bh = x.b * p.Hq + x.hk * group + g;
          const int st = (int)(n & 1u), qs = (int)(n % QST);
          const uint32_t ph = (n >> 1) & 1u, qph = (n / QST) & 1u;
          const long long srow = (long long)bh * p.S_pad + it * 128;
          if (!mbar_wait(&q_empty[qs], qph ^ 1u, abort_flag, kSiteBwdQDEmpty)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int cb = 0; cb < NB; ++cb) {
            mbar_arrive_expect_tx(&q_full[2 * qs + cb], 128 * 128 + (cb == NB - 1 ? Cfg::STATS_BYTES / 2 : 0));
            tma_load_3d(sQ + qs * TILE + cb * 128 * 128, &tmQ, &q_full[2 * qs + cb], cb * 64, it * 128, bh);
          }
          bulk_load(sLse + qs * 128, p.lse2 + srow, 512, &q_full[2 * qs + NB - 1]);
          qiss |= 1u << qs;
          qpar = (qpar & ~(1u << qs)) | (qph << qs);
          if (!mbar_wait(&do_empty[st], ph ^ 1u, abort_flag, kSiteBwdQDEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&do_full[st], TILE + Cfg::STATS_BYTES / 2);
          tma_load_rows<D>(sdO + st * TILE, &tmdO, &do_full[st], it * 128, bh);
          bulk_load(sDt + st * 128, p.dt + srow, 512, &do_full[st]);
          diss |= 1u << st;
          dpar = (dpar & ~(1u << st)) | (ph << st);
        }
      }
      if (!ok) {
        volatile int no_abort = 0;
        if (kviss) mbar_wait(kv_full, kvpar, &no_abort, kSiteBwdDrain);
        for (int s = 0; s < QST; ++s)
          if (qiss & (1u << s))
            for (int cb = 0; cb < NB; ++cb) mbar_wait(&q_full[2 * s + cb], (qpar >> s) & 1u, &no_abort, kSiteBwdDrain);
        for (int s = 0; s < 2; ++s)
          if (diss & (1u << s)) mbar_wait(&do_full[s], (dpar >> s) & 1u, &no_abort, kSiteBwdDrain);
      }
    } else if (warp == 1) {
      // ---------------------------------------------------------------- MMA issuer (whole warp, one elected lane issues)
      const bool leader = elect_one();
      constexpr uint32_t idesc_kv = make_idesc_f16(128, D, false, true);  // dV, dK: A in TMEM, B MN-major
      // descriptors built once; stages and K-steps are constant offsets from them
      const uint64_t k_desc = tile_desc_k(smem_u32(sK)), v_desc = tile_desc_k(smem_u32(sV));
      const uint64_t q_desc = tile_desc_k(smem_u32(sQ)), q_desc_mn = tile_desc_mn(smem_u32(sQ));
      const uint64_t do_desc = tile_desc_k(smem_u32(sdO)), do_desc_mn = tile_desc_mn(smem_u32(sdO));
      // dV += P^T dO or dK += dS^T Q: A at TMEM columns `a_col` + [64g, 64g+32) for g = 0, 1
      auto issue_kv = [&](uint32_t d_col, uint32_t a_col, uint64_t b_desc, bool first, int kk0 = 0, int kk1 = 8) {
#pragma unroll
        for (int kk = kk0; kk < kk1; ++kk) {  // 16 queries per K-step
          const uint32_t col = a_col + (uint32_t)(64 * (kk >> 2) + 8 * (kk & 3));
          if (leader)
            umma_f16_ts(tmem + d_col, tmem + col, sdesc_adv(b_desc, kk * 2048), idesc_kv, (!first || kk > 0) ? 1u : 0u);
        }
      };
      // S^T = K Q(n)^T from Q stage qs: each 64-column block's K-steps once that block landed
      auto issue_st = [&](uint32_t d_col, int qs, uint32_t par) -> bool {
        constexpr uint32_t idesc = make_idesc_f16(128, 128, false, false);
        const uint64_t qd = sdesc_adv(q_desc, qs * TILE);
#pragma unroll
        for (int cb = 0; cb < NB; ++cb) {
          if (!lane_wait(&q_full[2 * qs + cb], par, abort_flag, kSiteBwdQDFull)) return false;
          tc_fence_after();
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) {
            const uint32_t off = cb * 16384 + k4 * 32;
            if (leader) umma_f16_ss(tmem + d_col, sdesc_adv(k_desc, off), sdesc_adv(qd, off), idesc, (cb | k4) != 0 ? 1u : 0u);
          }
        }
        return true;
      };
      bool ok = true;
      // Tile cursors over the CTA's whole sequence of query tiles: `cur` is tile n, `nxt`
      // tile n + 1, possibly the first of the next item (read from the ring).
      int cur_ci = 0, cur_m = 0, nxt_ci = 0, nxt_m = 0;
      DkvItem cur = read_item(0, ok), nxt;
      auto advance = [&]() {  // nxt := the tile after cur
        nxt_ci = cur_ci;
        nxt_m = cur_m + 1;
        nxt = cur;
        if (nxt_m >= cur.n_iter) {
          nxt_ci = cur_ci + 1;
          nxt_m = 0;
          nxt = read_item(nxt_ci, ok);
        }
      };
      cur.valid = __all_sync(0xffffffffu, cur.valid && ok);
      if (cur.valid) {
        if (!warp_wait(kv_full, 0, abort_flag, kSiteBwdKV) || !issue_st(0, 0, 0) ||
            !warp_wait(&do_full[0], 0, abort_flag, kSiteBwdQDFull)) {
          ok = false;
        } else {
          tc_fence_after();
          if (leader) umma_commit(s_full);
          issue_score_tile<D>(leader, tmem + 128, v_desc, do_desc);
          if (leader) umma_commit(dp_full);
          if (cur.n_iter == 1 && leader) umma_commit(kv_empty);  // the item's last S^T / dP^T issued
          advance();
        }
      }
      for (uint32_t n = 0; cur.valid && ok; ++n) {
        const int st = (int)(n & 1u), st1 = (int)((n + 1) & 1u);
        const uint32_t par = n & 1u;
        const bool more = nxt.valid;  // the same on every lane: all read the same item
        const bool first = cur_m == 0;  // the item's first tile: dV and dK start afresh
        // ... in accumulators that may still hold the previous item's dV / dK: its dV / dK
        // MMAs then wait until the warps have read those out (acc_free)
        const bool defer = first && cur_ci > 0;
        const bool last = cur_m == cur.n_iter - 1;
        const uint32_t rs = (n & 1u) ? 128u : 0u, rp = 128u - rs;  // R_S(n), R_P(n)
        const int qs = (int)(n % QST), qs1 = (int)((n + 1) % QST);
        const uint64_t q_mn = sdesc_adv(q_desc_mn, qs * TILE), do_mn = sdesc_adv(do_desc_mn, st * TILE);
        // dV(n) as soon as P^T(n) is stored (the warps then wait for dP^T(n) and read it);
        // S^T(n+1) as soon as R_P(n) is free (the warps' next P phase waits for it); dK(n)
        // and dP^T(n+1) once dS^T(n) is stored, so dP^T(n+1) is done early in the next P phase.
        // (dV(n) in two halves around S^T(n+1): the issuing warp, which blocks while the
        // tensor pipe's queue is full, gets to S^T(n+1) sooner.)  Tile n+1 may be the next
        // item's first: its S^T / dP^T read the next item's K / V, which load once this
        // item's last S^T / dP^T have read K / V.  On an item's first tile the warps run the
        // P and dS phases before they write the previous item's dK / dV rows, so S^T(n+1) is
        // issued ahead of dV(n), which waits for acc_free; meanwhile the tensor core computes
        // S^T(n+1), and the warps' next P phase finds it ready.
        if (!lane_wait(p_ready, par, abort_flag, kSiteBwdDsFull)) break;
        tc_fence_after();
        if (!defer) issue_kv(T_DV, rs, do_mn, first, 0, 4);
        if (!lane_wait(rp_free, par, abort_flag, kSiteBwdDsFull)) break;
        if (more) {
          if (nxt_m == 0 && !lane_wait(kv_full, (uint32_t)nxt_ci & 1u, abort_flag, kSiteBwdKV)) break;
          if (!issue_st(rp, qs1, ((n + 1) / QST) & 1u)) break;
          if (leader) umma_commit(s_full);
        }
        if (defer) {
          if (!lane_wait(acc_free, (uint32_t)(cur_ci - 1) & 1u, abort_flag, kSiteBwdDkvFull)) break;
          tc_fence_after();
          issue_kv(T_DV, rs, do_mn, true, 0, 8);
        } else {
          issue_kv(T_DV, rs, do_mn, false, 4, 8);
        }
        if (!lane_wait(ds_ready, par, abort_flag, kSiteBwdDsFull)) break;
        tc_fence_after();
        // dO(n) read by dP^T(n) and dV(n), and Dt(n), which shares its stage, by the warps'
        // dS phase: the stage may take dO(n+2)
        if (leader) umma_commit(&do_empty[st]);
        issue_kv(T_DK, rs + 32, q_mn, first);
        if (leader) umma_commit(&q_empty[qs]);  // Q(n) read by S^T(n) and dK(n)
        if (last && leader) umma_commit(dkv_full);
        if (more) {  // into R_S(n), behind dV(n) and dK(n), which read P^T / dS^T(n) from it
          if (!lane_wait(&do_full[st1], ((n + 1) >> 1) & 1u, abort_flag, kSiteBwdQDFull)) break;
          tc_fence_after();
          issue_score_tile<D>(leader, tmem + rs, v_desc, sdesc_adv(do_desc, st1 * TILE));
          if (leader) umma_commit(dp_full);
          if (nxt_m == nxt.n_iter - 1 && leader) umma_commit(kv_empty);  // that item's last S^T / dP^T
        }
        if (last && leader) mbar_arrive(&item_empty[cur_ci % kDkvItemRing]);
        if (!more) break;
        cur = nxt;
        cur_ci = nxt_ci;
        cur_m = nxt_m;
        advance();
      }
      if (leader) umma_commit(drain);
      volatile int no_abort = 0;
      warp_wait(drain, 0, &no_abort, kSiteBwdDrain);
    }
  } else {
    warpgroup_reg_alloc<192>();
    // ---------------------------------------------------------------- softmax (warps 4..11)
    const uint32_t quarter = warp & 3u;
    const int g = (int)(warp - 4) >> 2;        // 64-query group / dV or dK (epilogue)
    const int r = (int)(quarter * 32 + lane);  // TMEM lane = key row
    const uint32_t lane_base = (quarter * 32u) << 16;
    bool ok = true;
    uint32_t n = 0;  // query tiles over all of the CTA's items
    // An item's dV (g = 0) / dK (g = 1) rows, 32-byte stores where the output allows (each a
    // whole sector of the row).  They are written after the next item's first P and dS
    // phases (the tensor core meanwhile computes that item's second S^T), and acc_free then
    // lets that item's dV / dK MMAs start the accumulators afresh.
    auto write_dkv = [&](const DkvItem& e, int eci) -> bool {
      if (!__all_sync(0xffffffffu, mbar_wait(dkv_full, (uint32_t)eci & 1u, abort_flag, kSiteBwdDkvFull)))
        return false;
      tc_fence_after();
      const int ekj = e.jt * 128 + r;
      const bool ekey_ok = ekj < p.S;
      const float sc = g == 0 ? 1.0f : p.scale;
      const uint32_t col = g == 0 ? T_DV : T_DK;
      __nv_bfloat16* orow = (g == 0 ? p.dv : p.dk) + ((long long)e.kvz * p.S + (ekey_ok ? ekj : 0)) * D;
      const bool o32 = (reinterpret_cast<uintptr_t>(g == 0 ? p.dv : p.dk) & 31u) == 0;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t a[32];
        tmem_ld32(tmem + lane_base + col + c * 32, a);
        tmem_wait_ld();
        if (ekey_ok) {
#pragma unroll
          for (int q = 0; q < 32; q += 16) {
            uint32_t wv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
              wv[i] = pack_bf16x2(__uint_as_float(a[q + 2 * i]) * sc, __uint_as_float(a[q + 2 * i + 1]) * sc);
            if (o32) {
              stg256(orow + c * 32 + q, wv[0], wv[1], wv[2], wv[3], wv[4], wv[5], wv[6], wv[7]);
            } else {  // only 16-byte aligned
              *reinterpret_cast<uint4*>(orow + c * 32 + q) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
              *reinterpret_cast<uint4*>(orow + c * 32 + q + 8) = make_uint4(wv[4], wv[5], wv[6], wv[7]);
            }
          }
        }
      }
      tc_fence_before();
      return true;
    };
    DkvItem prev;
    prev.valid = false;
    int prev_ci = 0;
    for (int ci = 0; ok; ++ci) {
      const DkvItem x = read_item(ci, ok);
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[ci % kDkvItemRing]);
      if (!__all_sync(0xffffffffu, ok && x.valid)) break;
      const int j0 = x.jt * 128;
      const int kj = j0 + r;
      const bool key_ok = kj < p.S;
      const bool keys_full = j0 + 128 <= p.S;
      for (int m = 0; m < x.n_iter && ok; ++m, ++n) {
        const int it = x.it0 + m % x.per_head;
        const int q0 = it * 128;
        const int st = (int)(n & 1u);
        const uint32_t par = n & 1u;
        const uint32_t rs = (n & 1u) ? 128u : 0u, rp = 128u - rs;
        // off-diagonal tiles need no mask: every key < S and every query >= every key
        const bool masked = !keys_full || (p.causal && it == x.jt);
        const int qmin = p.causal ? kj - q0 : -1;
        const int qs = (int)(n % QST);
        const uint32_t lse2_addr = smem_u32(sLse + qs * 128 + 64 * g), dt_addr = smem_u32(sDt + st * 128 + 64 * g);
        // first of this warp's 64 query columns that the key sees (64: none)
        const int first_ok = key_ok ? max(qmin - 64 * g, 0) : 64;
        // s_full: the scores; q_full: makes the TMA-written lse2 visible to this thread
        if (!__all_sync(0xffffffffu, mbar_wait(s_full, par, abort_flag, kSiteBwdStFull) &&
                                         mbar_wait(&q_full[2 * qs + NB - 1], (n / QST) & 1u, abort_flag,
                                                   kSiteBwdQDFull))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t cs = rs + 64 * g;  // this warp's 64 S^T columns
        float pe[64];
        {
          uint32_t sv[64];
          tmem_ld32(tmem + lane_base + cs, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
          tmem_ld32(tmem + lane_base + cs + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
          tmem_wait_ld();
          if (masked)
            bwd_p_cols<true>(sv, lse2_addr, p.scale_log2, first_ok, pe);
          else
            bwd_p_cols<false>(sv, lse2_addr, p.scale_log2, first_ok, pe);
          uint32_t pk[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) pk[i] = pack_bf16x2(pe[2 * i], pe[2 * i + 1]);
          tmem_st32(tmem + lane_base + cs, pk);  // P^T over the S^T columns just read
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_ready);
        // dp_full: dP^T(n); do_full: makes the TMA-written Dt visible to this thread
        if (!__all_sync(0xffffffffu, mbar_wait(dp_full, par, abort_flag, kSiteBwdStFull) &&
                                         mbar_wait(&do_full[st], (n >> 1) & 1u, abort_flag, kSiteBwdQDFull))) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t dpv[64];
        tmem_ld32(tmem + lane_base + rp + 64 * g, *reinterpret_cast<uint32_t(*)[32]>(&dpv[0]));
        tmem_ld32(tmem + lane_base + rp + 64 * g + 32, *reinterpret_cast<uint32_t(*)[32]>(&dpv[32]));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(rp_free);  // R_P(n) may take S^T(n+1)
        uint32_t dk[32];
#pragma unroll
        for (int e4 = 0; e4 < 16; ++e4) {
          const float4 d4 = lds_f4(dt_addr + 16 * e4);
          const float dv[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
          for (int u = 0; u < 4; u += 2) {
            const int e = 4 * e4 + u;
            float t0, t1, d0, d1;
            fma2(t0, t1, dv[u], dv[u + 1], -1.0f, -1.0f, __uint_as_float(dpv[e]), __uint_as_float(dpv[e + 1]));
            mul2(d0, d1, pe[e], pe[e + 1], t0, t1);
            dk[e >> 1] = pack_bf16x2(d0, d1);
          }
        }
        tmem_st32(tmem + lane_base + cs + 32, dk);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(ds_ready);
        if (m == 0 && prev.valid) {  // the previous item's rows, then its accumulators are free
          if (!write_dkv(prev, prev_ci)) {
            ok = false;
            break;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(acc_free);
          prev.valid = false;
        }
      }
      if (!ok) break;
      prev = x;
      prev_ci = ci;
    }
    // the CTA's last item
    if (ok && prev.valid) write_dkv(prev, prev_ci);
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) sched_finish(p.sched_slot);  // every fetch of this CTA is done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// 3. dQ.  Persistent: one CTA per SM walks work items (128-query tile, query head),
//    heaviest causal tiles first; its first item is w = blockIdx.x, the next ones come from
//    the launch's work counter (sched_fetch), so the CTAs finish together although items
//    differ in cost by up to 32x.  The producer fetches and publishes each item in a
//    four-slot ring in shared memory (item_full / item_empty), read by the MMA warp and
//    the softmax warps.  Per key tile of
//    an item (thread = query row, so lse2 and Dt are per-thread registers):
//   S(t)  = Q K_j^T -> TMEM [128 (t&1), +128)  (double-buffered: S(t+1) is computed while
//                                               the warps work on tile t)
//   dP(t) = dO V_j^T -> TMEM [256,384)          (issued once every warp holds dP(t-1))
//   softmax warp (g, quarter): query rows 32*quarter.., key columns 64g..64g+63 in two
//   chunks; dS = P (dP - Dt), P = exp2(S * scale*log2e - lse2), bf16 -> TMEM over the S
//   columns already read, then  dQ += dS K_j  with A read from TMEM.
//   t counts key tiles over all of the CTA's items, so the rings, the S buffers and the
//   barrier phases run on across items: the next item's S and dP are computed while the
//   warps finish the current one and store its dQ, and its Q (dO) loads as soon as the
//   current item's last S (dP) has read Q (dO).  The first dQ MMA of an item waits until
//   the warps have read the previous item's dQ out of TMEM.
// TMEM: S [0,256) | dP [256,384) | dQ [384,384+D).
// ---------------------------------------------------------------------------
struct DqItem {
  bool valid;
  int w, ci, j, n_kt, it, bh, kvz;
};

// Work item `w` (the ci-th of this CTA), positioned at its key tile 0; w at or beyond the
// item count is the end of the CTA's work.
__device__ __forceinline__ DqItem dq_item(const AttnBwdParams& p, int w, int ci) {
  DqItem x;
  const int n_bh = p.B * p.Hq, n_qt = (p.S + 127) / 128;
  x.valid = w < n_qt * n_bh;
  x.w = w;
  x.ci = ci;
  x.j = 0;
  // grouped head order (K/V tiles re-read from L2), the last query tile (most causal work)
  // first
  if (x.valid) {
    grouped_order(w, n_bh, n_qt, x.it, x.bh);
    x.it = n_qt - 1 - x.it;
  } else {
    x.it = 0;
    x.bh = 0;
  }
  x.kvz = (x.bh / p.Hq) * p.Hkv + (x.bh % p.Hq) / (p.Hq / p.Hkv);
  x.n_kt = p.causal ? x.it + 1 : n_qt;
  return x;
}

constexpr int kDqItemRing = 4;

template <int D>
__global__ void __launch_bounds__(384, 1)
    k_attn_bwd_dq(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                  const AttnBwdParams p) {
  using Cfg = AttnBwdCfg<D>;
  constexpr uint32_t TILE = Cfg::TILE_BYTES;
  constexpr int KST = 3;  // K ring depth: S(t+2) is issued while K(t), K(t+1) are in use
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sdO = sQ + TILE;
  uint8_t* sK = sdO + TILE;       // [3]
  uint8_t* sV = sK + KST * TILE;  // [2]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + 2 * TILE);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [3]
  uint64_t* k_empty = bars + 4;   // [3]
  uint64_t* v_full = bars + 7;    // [2]
  uint64_t* v_empty = bars + 9;   // [2]
  uint64_t* s_full = bars + 11;   // [2] S(t) and dP(t) computed, by S buffer
  uint64_t* dp_free = bars + 13;  // dP(t) read by all 8 warps
  // [chunk][tile parity]: dS chunk c of tile t stored by all 8 warps.  By tile parity
  // because the warps may store tile t+1's chunks (S(t+1) and dP(t+1) are issued before
  // the MMA warp waits for tile t's) before the MMA warp has seen tile t's.
  uint64_t* ds_chunk = bars + 14;  // [2][2]
  uint64_t* dq_full = bars + 18;   // an item's dQ complete
  uint64_t* drain = bars + 19;
  uint64_t* q_empty = bars + 20;   // Q read by the item's last S
  uint64_t* do_full = bars + 21;
  uint64_t* do_empty = bars + 22;  // dO read by the item's last dP
  uint64_t* dq_free = bars + 23;   // an item's dQ read out of TMEM by all 8 warps
  uint64_t* item_full = bars + 24;                 // [4] item published by the producer
  uint64_t* item_empty = item_full + kDqItemRing;  // [4] read by the MMA warp and the 8 softmax warps
  int* s_item = reinterpret_cast<int*>(item_empty + kDqItemRing);  // [4] item indices
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_item + kDqItemRing);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  constexpr uint32_t T_S = 0, T_DP = 256, T_DQ = 384;

  const uint32_t warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    mbar_init(do_full, 1);
    mbar_init(do_empty, 1);
    for (int i = 0; i < KST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&ds_chunk[i], 8);
      mbar_init(&ds_chunk[2 + i], 8);
    }
    mbar_init(dp_free, 8);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 8);
    mbar_init(drain, 1);
    for (int i = 0; i < kDqItemRing; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 9);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  // The ci-th item of this CTA, from the ring (every role but the producer).
  auto read_item = [&](int ci, bool& ok) -> DqItem {
    const int slot = ci % kDqItemRing;
    if (!mbar_wait(&item_full[slot], (uint32_t)(ci / kDqItemRing) & 1u, abort_flag, kSiteQItem)) {
      ok = false;
      return dq_item(p, INT32_MAX, ci);
    }
    return dq_item(p, s_item[slot], ci);
  };
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    warpgroup_reg_dealloc<120>();
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------------------- producer
      // per item: Q, then K/V of its key tiles with dO after the first K/V pair (the first
      // S needs Q and K, the first dP dO and V)
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmdO);
      uint32_t kiss = 0, viss = 0, kpar = 0, vpar = 0, qiss = 0, qpar = 0, diss = 0, dpar = 0;
      bool ok = true;
      uint32_t t = 0;
      const int n_items = p.B * p.Hq * ((p.S + 127) / 128);
      for (int ci = 0; ok; ++ci) {
        // fetch the CTA's next item and publish it (an index >= n_items ends every role)
        const int w = ci == 0 ? (int)blockIdx.x : sched_fetch(p.sched_slot);
        const int slot = ci % kDqItemRing;
        if (!mbar_wait(&item_empty[slot], ((uint32_t)(ci / kDqItemRing) & 1u) ^ 1u, abort_flag, kSiteQItem)) {
          ok = false;
          break;
        }
        s_item[slot] = w < n_items ? w : n_items;
        mbar_arrive(&item_full[slot]);
        const DqItem x = dq_item(p, w, ci);
        if (!x.valid) break;
        const uint32_t iph = (uint32_t)x.ci & 1u;
        if (!mbar_wait(q_empty, iph ^ 1u, abort_flag, kSiteQKEmpty)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(q_full, TILE);
        tma_load_rows<D>(sQ, &tmQ, q_full, x.it * 128, x.bh);
        qiss = 1;
        qpar = iph;
        for (int j = 0; j < x.n_kt; ++j, ++t) {
          const int ks = (int)(t % KST), vs = (int)(t & 1);
          const uint32_t kph = (t / KST) & 1u, vph = (t >> 1) & 1u;
          if (!mbar_wait(&k_empty[ks], kph ^ 1u, abort_flag, kSiteQKEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[ks], TILE);
          tma_load_rows<D>(sK + ks * TILE, &tmK, &k_full[ks], j * 128, x.kvz);
          kiss |= 1u << ks;
          kpar = (kpar & ~(1u << ks)) | (kph << ks);
          if (!mbar_wait(&v_empty[vs], vph ^ 1u, abort_flag, kSiteQVEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&v_full[vs], TILE);
          tma_load_rows<D>(sV + vs * TILE, &tmV, &v_full[vs], j * 128, x.kvz);
          viss |= 1u << vs;
          vpar = (vpar & ~(1u << vs)) | (vph << vs);
          if (j == 0) {
            if (!mbar_wait(do_empty, iph ^ 1u, abort_flag, kSiteQVEmpty)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(do_full, TILE);
            tma_load_rows<D>(sdO, &tmdO, do_full, x.it * 128, x.bh);
            diss = 1;
            dpar = iph;
          }
        }
      }
      if (!ok) {
        volatile int no_abort = 0;
        if (qiss) mbar_wait(q_full, qpar, &no_abort, kSiteQDrain);
        if (diss) mbar_wait(do_full, dpar, &no_abort, kSiteQDrain);
        for (int s = 0; s < KST; ++s)
          if (kiss & (1u << s)) mbar_wait(&k_full[s], (kpar >> s) & 1u, &no_abort, kSiteQDrain);
        for (int s = 0; s < 2; ++s)
          if (viss & (1u << s)) mbar_wait(&v_full[s], (vpar >> s) & 1u, &no_abort, kSiteQDrain);
      }
    } else if (warp == 1) {
      // ---------------------------------------------------------------- MMA issuer (whole warp, one elected lane issues)
      const bool leader = elect_one();
      constexpr uint32_t idesc_q = make_idesc_f16(128, D, false, true);  // dQ: A = dS in TMEM, B = K MN-major
      const uint64_t q_desc = tile_desc_k(smem_u32(sQ)), do_desc = tile_desc_k(smem_u32(sdO));
      const uint64_t k_desc = tile_desc_k(smem_u32(sK)), k_desc_mn = tile_desc_mn(smem_u32(sK));
      const uint64_t v_desc = tile_desc_k(smem_u32(sV));
      auto issue_s = [&](const DqItem& x, uint32_t t) -> bool {  // S(t) into buffer t&1
        if (x.j == 0 && !lane_wait(q_full, (uint32_t)x.ci & 1u, abort_flag, kSiteQQd)) return false;
        if (!lane_wait(&k_full[t % KST], (t / KST) & 1u, abort_flag, kSiteQKFull)) return false;
        tc_fence_after();
        issue_score_tile<D>(leader, tmem + T_S + 128 * (t & 1), q_desc, sdesc_adv(k_desc, (t % KST) * TILE));
        if (x.j == x.n_kt - 1 && leader) umma_commit(q_empty);  // the item's last S has read Q
        return true;
      };
      auto issue_dp = [&](const DqItem& x, uint32_t t) -> bool {  // dP(t); then S(t) and dP(t) are announced
        if (x.j == 0 && !lane_wait(do_full, (uint32_t)x.ci & 1u, abort_flag, kSiteQQd)) return false;
        if (!lane_wait(&v_full[t & 1], (t >> 1) & 1u, abort_flag, kSiteQVFull)) return false;
        tc_fence_after();
        issue_score_tile<D>(leader, tmem + T_DP, do_desc, sdesc_adv(v_desc, (t & 1) * TILE));
        if (leader) umma_commit(&v_empty[t & 1]);
        if (leader) umma_commit(&s_full[t & 1]);
        if (x.j == x.n_kt - 1 && leader) umma_commit(do_empty);  // the item's last dP has read dO
        return true;
      };
      bool ok = true;
      // The key tile after `x`: the next tile of the item, or tile 0 of the CTA's next item
      // (read from the ring: the leading cursor waits for it, the others find it there).  The
      // end of the CTA's work stays the end: no slot is published after it.
      auto dq_next = [&](DqItem x) -> DqItem {
        if (!x.valid || ++x.j < x.n_kt) return x;
        return read_item(x.ci + 1, ok);
      };
      DqItem xq = read_item(0, ok);  // tile t: dQ
      DqItem xp = xq, xs = xq;       // tiles t+1: dP, t+2: S
      if (xs.valid) {
        ok = issue_s(xs, 0) && issue_dp(xp, 0);
        xs = dq_next(xs);
        xp = dq_next(xp);
        if (ok && xs.valid) ok = issue_s(xs, 1);
        xs = dq_next(xs);
      }
      for (uint32_t t = 0; xq.valid && ok; ++t) {
        const uint32_t sb = T_S + 128 * (t & 1);
        const uint64_t k_mn = sdesc_adv(k_desc_mn, (t % KST) * TILE);
        if (!lane_wait(dp_free, t & 1u, abort_flag, kSiteQDpFree)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (xp.valid) {
          if (!issue_dp(xp, t + 1)) {
            ok = false;
            break;
          }
          xp = dq_next(xp);
        }
        // the item's first dQ MMA overwrites the accumulator: the previous item's dQ must be out
        if (xq.j == 0 && xq.ci > 0 && !lane_wait(dq_free, (uint32_t)(xq.ci - 1) & 1u, abort_flag, kSiteQDqFull)) {
          ok = false;
          break;
        }
        for (int c = 0; c < 2 && ok; ++c) {
          if (!lane_wait(&ds_chunk[2 * c + (t & 1)], (t >> 1) & 1u, abort_flag, kSiteQDsFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int i = 0; i < 4; ++i) {  // this chunk's K-steps: 16 keys each
            const int kk = (i >> 1) * 4 + 2 * c + (i & 1);
            const uint32_t acc = (xq.j > 0 || c > 0 || i > 0) ? 1u : 0u;
            if (leader) umma_f16_ts(tmem + T_DQ, tmem + sb + (uint32_t)((kk >> 2) * 64 + (kk & 3) * 8),
                                    sdesc_adv(k_mn, kk * 2048), idesc_q, acc);
          }
        }
        if (!ok) break;
        if (leader) umma_commit(&k_empty[t % KST]);  // K(t) read by S(t) and dQ(t)
        if (xq.j == xq.n_kt - 1 && leader) umma_commit(dq_full);
        if (xs.valid) {  // behind dQ(t), which read dS(t) from that buffer
          if (!issue_s(xs, t + 2)) {
            ok = false;
            break;
          }
          xs = dq_next(xs);
        }
        // the dQ cursor leaves its item: the MMA warp is done with the ring slot
        if (xq.j == xq.n_kt - 1 && leader) mbar_arrive(&item_empty[xq.ci % kDqItemRing]);
        xq = dq_next(xq);
      }
      if (leader) umma_commit(drain);
      volatile int no_abort = 0;
      warp_wait(drain, 0, &no_abort, kSiteQDrain);
    }
  } else {
    warpgroup_reg_alloc<192>();
    // ---------------------------------------------------------------- softmax (warps 4..11)
    const uint32_t quarter = warp & 3u;
    const int g = (int)(warp - 4) >> 2;        // key-column half (softmax) / head-dim half (epilogue)
    const int r = (int)(quarter * 32 + lane);  // TMEM lane = query row
    const uint32_t lane_base = (quarter * 32u) << 16;
    bool ok = true;
    uint32_t t = 0;
    for (int ci = 0; ok; ++ci) {
      const DqItem x = read_item(ci, ok);
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[ci % kDqItemRing]);
      if (!__all_sync(0xffffffffu, ok) || !x.valid) break;
      const int qi = x.it * 128 + r;
      const long long srow = (long long)x.bh * p.S_pad + qi;  // padded rows: -lse2 = -inf, Dt = 0
      const float nl2 = __ldg(p.lse2 + srow), dtr = __ldg(p.dt + srow);
      for (int j = 0; j < x.n_kt; ++j, ++t) {
        const uint32_t sb = T_S + 128 * (t & 1) + 64 * g;
        const int k0 = j * 128 + 64 * g;
        // keys at or beyond S, and (causal) keys after the query, are masked
        const bool masked = (k0 + 64 > p.S) || (p.causal && j == x.it);
        const int klim = p.causal ? min(p.S - k0, qi - k0 + 1) : p.S - k0;
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[t & 1], (t >> 1) & 1u, abort_flag, kSiteQSFull))) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t s[2][32], dp[2][32];
        tmem_ld32(tmem + lane_base + sb, s[0]);
        tmem_ld32(tmem + lane_base + T_DP + 64 * g, dp[0]);
        tmem_ld32(tmem + lane_base + sb + 32, s[1]);
        tmem_ld32(tmem + lane_base + T_DP + 64 * g + 32, dp[1]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dp_free);  // dP(t+1) may overwrite dP(t)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[16];
          if (masked)
            dq_ds_chunk<true>(s[c], dp[c], p.scale_log2, nl2, dtr, klim - 32 * c, pk);
          else
            dq_ds_chunk<false>(s[c], dp[c], p.scale_log2, nl2, dtr, klim - 32 * c, pk);
          tmem_st16(tmem + lane_base + sb + 16 * c, pk);  // over S columns this thread has read
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&ds_chunk[2 * c + (t & 1)]);
        }
      }
      if (!ok) break;
      // dQ rows: this warp stores head-dim columns [g D/2, (g+1) D/2)
      if (!__all_sync(0xffffffffu, mbar_wait(dq_full, (uint32_t)x.ci & 1u, abort_flag, kSiteQDqFull))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t a[D / 64][32];
#pragma unroll
      for (int c = 0; c < D / 64; ++c) tmem_ld32(tmem + lane_base + T_DQ + g * (D / 2) + c * 32, a[c]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free);  // the next item's dQ may start
      if (qi < p.S) {  // 32-byte stores where dQ allows: each fills a whole sector of the row
        const bool dq32 = (reinterpret_cast<uintptr_t>(p.dq) & 31u) == 0;
        __nv_bfloat16* row = p.dq + ((long long)x.bh * p.S + qi) * D + g * (D / 2);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
#pragma unroll
          for (int e = 0; e < 32; e += 16) {
            uint32_t w[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
              w[i] = pack_bf16x2(__uint_as_float(a[c][e + 2 * i]) * p.scale, __uint_as_float(a[c][e + 2 * i + 1]) * p.scale);
            if (dq32) {
              stg256(row + c * 32 + e, w[0], w[1], w[2], w[3], w[4], w[5], w[6], w[7]);
            } else {  // dQ only 16-byte aligned
              *reinterpret_cast<uint4*>(row + c * 32 + e) = make_uint4(w[0], w[1], w[2], w[3]);
              *reinterpret_cast<uint4*>(row + c * 32 + e + 8) = make_uint4(w[4], w[5], w[6], w[7]);
            }
          }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) sched_finish(p.sched_slot);  // every fetch of this CTA is done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

}  // namespace beacon
