// attention.cuh -- causal scaled-dot-product attention forward on tcgen05 tensor cores.
//
// Kernel ID `attention_adjoint_fwd` (crates/beacon-cuda/src/attention.rs:21-40).
// Persistent: one CTA per SM walks work items (pair of 128-row query tiles, batch*head),
// its first item its block index and the next ones from the launch's work counter, so
// the SMs finish together although causal items differ in cost by up to the number of
// key tiles.  The rings, TMEM regions and barrier phases run on across items: the next
// item's Q loads as soon as the current item's last S has read Q, and its first S MMAs
// follow the last PV MMAs at once, running while the softmax warps write the item's
// output (one CTA per item spent ~5k cycles before its first S and ~6k after its last).
// The two tiles (A, B) of an item share every K/V tile and ping-pong on the tensor core:
// while one softmax warpgroup turns S_A into P_A, the tensor core computes S_B, and so on:
//
//   MMA issue order:   S_A(0) S_B(0) | O_A += P_A(j) V_j, S_A(j+1), O_B += P_B(j) V_j, S_B(j+1) | ...
//
// with each PV product issued in two 64-key halves, each as soon as the softmax warps have
// stored that half of P, so the tensor core starts on P while the warps finish it.
//
//   warp 0      TMA producer: fetches and publishes the work items (a four-slot ring in
//               shared memory); per item Q_A, Q_B, then K_j and V_j into 2-deep rings.
//   warp 1      TMEM allocator + tcgen05.mma issuer (the whole warp runs the issue loop,
//               one elected lane issues).
//   warps 2-3   idle; warps 0-3 hand most of their registers to the softmax warpgroups
//               (setmaxnreg), so a thread holds its whole S row without spilling.
//   warps 4-7   softmax of tile A, warps 8-11 softmax of tile B: one query row per
//               thread (TMEM lane = row), online softmax in the log2 domain with fp32
//               statistics.  P (bf16) is written back into the first 64 TMEM columns
//               of its own S region and read from there as the A operand of the PV
//               MMA, so P never touches shared memory.  O is rescaled in TMEM only
//               when a row maximum grows by more than 2^8 (P and l share the stale
//               maximum, so O / l is exact either way).
//
// TMEM: S_A [0,128), S_B [128,256), O_A [256,256+D), O_B [256+D,256+2D).
//
// RECOMP = true is the forward the drop-in backward runs, given the saved LSE: P =
// exp2(S * scale*log2e - lse*log2e) is final as it is computed (no running maximum, no
// rescale, no row sum), O accumulates already normalised, and the epilogue writes the
// backward's row statistics instead of O: Dt = rowsum(dO * O) (O in fp32 from TMEM, dO
// read from global memory) and lse2 = -lse*log2e, both padded to whole 128-row tiles
// (0 / -inf on rows at or beyond S).
#pragma once

#include "sm100.cuh"

namespace beacon {

struct AttnParams {
  int B, Hq, Hkv, S;
  float scale_log2;  // softmax scale * log2(e)
  int causal;
  __nv_bfloat16* out;  // [B, Hq, S, D]
  float* lse;          // [B, Hq, S]
  int n_qtiles;
  int n_pairs;         // ceil(n_qtiles / 2)
  int out_tokens;      // 1: out is token-major [B, S, Hq, D] (the input of an output projection)
  int sched_slot;      // the launch's work counter (g_sched)
  // RECOMP only
  const float* lse_in;            // [B, Hq, S] saved LSE (natural log)
  const __nv_bfloat16* dout;      // [B, Hq, S, D]
  float* dt;                      // [B*Hq, S_pad] rowsum(dO * O)
  float* lse2;                    // [B*Hq, S_pad] -lse * log2(e)
  int S_pad;
};

template <int D>
struct AttnFwdCfg {
  static constexpr int BM = 128, BN = 128;
  static constexpr uint32_t Q_BYTES = BM * D * 2;
  static constexpr uint32_t KV_BYTES = BN * D * 2;
  static constexpr size_t SMEM_BYTES = 1024 + 2 * (size_t)Q_BYTES + 4 * (size_t)KV_BYTES + 512;
  static constexpr int THREADS = 384;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t S_COL_STRIDE = 128;  // S_A at column 0, S_B at column 128
  static constexpr uint32_t O_COL0 = 256;
};

enum : unsigned int {
  kSiteAttnQ = 0x201,
  kSiteAttnKFull = 0x202,
  kSiteAttnKEmpty = 0x203,
  kSiteAttnVFull = 0x204,
  kSiteAttnVEmpty = 0x205,
  kSiteAttnSFull = 0x206,
  kSiteAttnPvDone = 0x207,
  kSiteAttnPFull = 0x208,
  kSiteAttnOFull = 0x20a,
  kSiteAttnDrain = 0x20b,
  kSiteAttnItem = 0x20c,
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Work order of the attention kernels: heads in groups of kHeadGroup; within a group the
// heaviest causal tiles of all its heads first (rank 0 = heaviest), then the next rank.
// The CTAs in flight then share few heads, so K/V (or Q/dO) tiles come from HBM about once
// and from L2 after that, and each group still ends with its lightest tiles (a balanced
// tail).  Linear index w -> (rank, head) for `n_heads` heads of `n_ranks` tiles each.
constexpr int kHeadGroup = 8;
__device__ __forceinline__ void grouped_order(int w, int n_heads, int n_ranks, int& rank, int& head) {
  const int per_group = kHeadGroup * n_ranks;
  const int g = w / per_group, base = g * kHeadGroup;
  const int in_group = min(kHeadGroup, n_heads - base);
  const int r = w - g * per_group;
  rank = r / in_group;
  head = base + r % in_group;
}

// Loads one 128-row x D tile (rows `row0..row0+127` of head `z`) as D/64 swizzled
// column blocks of 128 rows x 128 bytes.
template <int D>
__device__ __forceinline__ void tma_load_rows(uint8_t* dst, const CUtensorMap* m, uint64_t* bar, int row0, int z) {
#pragma unroll
  for (int b = 0; b < D / 64; ++b) tma_load_3d(dst + b * 128 * 128, m, bar, b * 64, row0, z);
}

// 2^a for a pair of arguments without the MUFU unit: a = n + f with n = rint(a) (1.5 x 2^23
// added and subtracted in fp32 round-to-nearest, n then sits in the low mantissa bits),
// a cubic in f in [-0.5, 0.5] fitted to 2^f by iteratively reweighted least squares on the
// relative error (max relative error 7.5e-5 on [-125.5, 8], far below the bf16 rounding P receives), and n
// shifted into the exponent field.  Arguments are clamped at -126, which returns less than
// 2^-125 instead of 0, so callers use it only where no element is masked to -inf.
__device__ __forceinline__ void exp2_poly2(float& r0, float& r1, float a0, float a1) {
  constexpr float kMagic = 12582912.0f;
  a0 = fmaxf(a0, -126.0f);
  a1 = fmaxf(a1, -126.0f);
  float t0, t1, n0, n1, f0, f1, p0, p1;
  add2(t0, t1, a0, a1, kMagic, kMagic);
  add2(n0, n1, t0, t1, -kMagic, -kMagic);
  fma2(f0, f1, n0, n1, -1.0f, -1.0f, a0, a1);
  fma2(p0, p1, 5.5171408e-2f, 5.5171408e-2f, f0, f1, 2.4261075e-1f, 2.4261075e-1f);
  fma2(p0, p1, p0, p1, f0, f1, 6.9326097e-1f, 6.9326097e-1f);
  fma2(p0, p1, p0, p1, f0, f1, 9.9992812e-1f, 9.9992812e-1f);
  r0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  r1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

// Pairs of S columns whose exponentials run on the FMA pipe on unmasked tiles, one bit per
// pair index mod 8: the exponential unit (16 results per clock per SM) and the FMA pipe
// then finish the row in about the same time.  (A quarter measured fastest: three or four
// eighths on the FMA pipe were 3-4% slower.)
constexpr uint32_t kPolyPairs = 0x11u;

// P = 2^(x * scale_log2 - m) for one 128-wide S row, packed to bf16 pairs into the
// 64 TMEM columns at `taddr`; returns the row sum of P (fp32, before rounding).  The
// argument and the running sums use packed f32x2 instructions.
// After each 64-key half is stored, the warp arrives on p_half[half]: the PV MMA of that
// half starts while the warp works on the other.
template <bool POLY>
__device__ __forceinline__ float softmax_p_to_tmem(const float* x, float scale_log2, float neg_m, uint32_t taddr,
                                                   uint64_t* p_half) {
  float ls[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t pk[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      float a0, a1, p0, p1;
      fma2(a0, a1, x[64 * c + 2 * e], x[64 * c + 2 * e + 1], scale_log2, scale_log2, neg_m, neg_m);
      if (POLY && ((kPolyPairs >> (e & 7)) & 1u)) {
        exp2_poly2(p0, p1, a0, a1);
      } else {
        p0 = ex2_approx(a0);
        p1 = ex2_approx(a1);
      }
      const int q = 2 * (e & 1);
      add2(ls[q], ls[q + 1], ls[q], ls[q + 1], p0, p1);
      pk[e] = pack_bf16x2(p0, p1);
    }
    tmem_st32(taddr + 32 * c, pk);
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane_id() == 0) mbar_arrive(&p_half[c]);
  }
  return (ls[0] + ls[1]) + (ls[2] + ls[3]);
}

// Work items of the persistent forward: (pair of query tiles, batch*head) in the grouped
// head order, the heaviest causal pairs of a group first.  Published by the producer in a
// four-slot ring in shared memory.
constexpr int kFwdItemRing = 4;
struct FwdItem {
  bool valid;
  int bh, kvz, n_j;
  int q0[2], nkv[2];  // per tile: first query row, key tiles it attends to (0: tile beyond S)
};
__device__ __forceinline__ FwdItem fwd_item(const AttnParams& p, int w, int n_bh, int n_ktiles) {
  FwdItem x;
  x.valid = w < p.n_pairs * n_bh;
  int pair = 0, bh = 0;
  if (x.valid) {
    grouped_order(w, n_bh, p.n_pairs, pair, bh);
    pair = p.n_pairs - 1 - pair;
  }
  x.bh = bh;
  x.kvz = (bh / p.Hq) * p.Hkv + (bh % p.Hq) / (p.Hq / p.Hkv);
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int qt = 2 * pair + t;
    x.q0[t] = qt * 128;
    x.nkv[t] = (!x.valid || x.q0[t] >= p.S) ? 0 : (p.causal ? min(qt + 1, n_ktiles) : n_ktiles);
  }
  x.n_j = max(x.nkv[0], x.nkv[1]);
  return x;
}

template <int D, bool RECOMP = false>
__global__ void __launch_bounds__(384, 1)
    k_attn_fwd_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using Cfg = AttnFwdCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                      // [2] tiles A, B
  uint8_t* sK = sQ + 2 * Cfg::Q_BYTES;     // [2] stages
  uint8_t* sV = sK + 2 * Cfg::KV_BYTES;    // [2] stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + 2 * Cfg::KV_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* v_full = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [2] per tile
  uint64_t* p_full = bars + 11;   // [2][2] per tile and 64-key half: P stored by its 4 warps
  uint64_t* o_full = bars + 15;   // [2] per tile
  uint64_t* drain = bars + 17;
  uint64_t* q_empty = bars + 18;                    // Q_A, Q_B read by the item's last S
  uint64_t* item_full = bars + 19;                  // [4] item published by the producer
  uint64_t* item_empty = item_full + kFwdItemRing;  // [4] read by the MMA warp and the 8 softmax warps
  int* s_item = reinterpret_cast<int*>(item_empty + kFwdItemRing);  // [4] item indices
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_item + kFwdItemRing);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id(), lane = lane_id();
  const int n_bh = p.B * p.Hq;
  const int n_items = p.n_pairs * n_bh;
  const int n_ktiles = (p.S + Cfg::BN - 1) / Cfg::BN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[2 * i], 4);
      mbar_init(&p_full[2 * i + 1], 4);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < kFwdItemRing; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 9);
    }
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

  // The ci-th item of this CTA from the ring (every role but the producer): false at the
  // end of the CTA's work or when a wait gave up.
  auto read_item = [&](int ci, FwdItem& x) -> bool {
    const int slot = ci % kFwdItemRing;
    if (!mbar_wait(&item_full[slot], (uint32_t)(ci / kFwdItemRing) & 1u, abort_flag, kSiteAttnItem)) return false;
    x = fwd_item(p, s_item[slot], n_bh, n_ktiles);
    return x.valid;
  };

  // Registers: the producer / MMA warpgroup gives up most of its share to the two
  // softmax warpgroups, which hold a whole 128-column S row per thread.
  // 128 x 72 + 256 x 216 = 384 x 168, the allocation the CTA is launched with.
  if (warp < 4) {
    warpgroup_reg_dealloc<72>();
    if (warp == 0) {
      // ---------------------------------------------------------------- producer
      if (lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        // K/V tiles are counted over all of the CTA's items (tk): the rings run on across items
        uint32_t tk = 0, kissued = 0, vissued = 0, kpar = 0, vpar = 0, qissued = 0, qpar = 0;
        bool ok = true;
        for (int ci = 0; ok; ++ci) {
          // fetch the CTA's next item and publish it (an index >= n_items ends every role)
          const int w = ci == 0 ? (int)blockIdx.x : sched_fetch(p.sched_slot);
          const int slot = ci % kFwdItemRing;
          if (!mbar_wait(&item_empty[slot], ((uint32_t)(ci / kFwdItemRing) & 1u) ^ 1u, abort_flag, kSiteAttnItem)) {
            ok = false;
            break;
          }
          s_item[slot] = w < n_items ? w : n_items;
          mbar_arrive(&item_full[slot]);
          const FwdItem x = fwd_item(p, w, n_bh, n_ktiles);
          if (!x.valid) break;
          // Q_A, Q_B once the previous item's last S has read them
          if (!mbar_wait(q_empty, ((uint32_t)ci & 1u) ^ 1u, abort_flag, kSiteAttnQ)) { ok = false; break; }
          mbar_arrive_expect_tx(q_full, 2 * Cfg::Q_BYTES);
          tma_load_rows<D>(sQ, &tmQ, q_full, x.q0[0], x.bh);
          tma_load_rows<D>(sQ + Cfg::Q_BYTES, &tmQ, q_full, x.q0[1], x.bh);  // rows >= S read as zeros
          qissued = 1;
          qpar = (uint32_t)ci & 1u;
          for (int j = 0; j < x.n_j; ++j, ++tk) {
            const int st = (int)(tk & 1u);
            const uint32_t ph = (tk >> 1) & 1u;
            if (!mbar_wait(&k_empty[st], ph ^ 1u, abort_flag, kSiteAttnKEmpty)) { ok = false; break; }
            mbar_arrive_expect_tx(&k_full[st], Cfg::KV_BYTES);
            tma_load_rows<D>(sK + st * Cfg::KV_BYTES, &tmK, &k_full[st], j * Cfg::BN, x.kvz);
            kissued |= 1u << st;
            kpar = (kpar & ~(1u << st)) | (ph << st);
            if (!mbar_wait(&v_empty[st], ph ^ 1u, abort_flag, kSiteAttnVEmpty)) { ok = false; break; }
            mbar_arrive_expect_tx(&v_full[st], Cfg::KV_BYTES);
            tma_load_rows<D>(sV + st * Cfg::KV_BYTES, &tmV, &v_full[st], j * Cfg::BN, x.kvz);
            vissued |= 1u << st;
            vpar = (vpar & ~(1u << st)) | (ph << st);
          }
        }
        if (!ok) {
          volatile int no_abort = 0;
          if (qissued) mbar_wait(q_full, qpar, &no_abort, kSiteAttnDrain);
          for (int s = 0; s < 2; ++s) {
            if (kissued & (1u << s)) mbar_wait(&k_full[s], (kpar >> s) & 1u, &no_abort, kSiteAttnDrain);
            if (vissued & (1u << s)) mbar_wait(&v_full[s], (vpar >> s) & 1u, &no_abort, kSiteAttnDrain);
          }
        }
      }
    } else if (warp == 1) {
      // ---------------------------------------------------------------- MMA issuer (whole warp, one elected lane issues)
      {
        const bool leader = elect_one();
        constexpr uint32_t idesc_s = make_idesc_f16(128, 128, false, false);
        constexpr uint32_t idesc_o = make_idesc_f16(128, D, false, true);
        // descriptors built once; tiles, stages and K-steps are constant offsets from them
        const uint64_t q_desc = make_sdesc_sw128(smem_u32(sQ), 16, 1024);
        const uint64_t k_desc = make_sdesc_sw128(smem_u32(sK), 16, 1024);
        const uint64_t v_desc = make_sdesc_sw128(smem_u32(sV), 128 * 128, 1024);
        // S_t(j) = Q_t K^T (K tile of ring count `tk`) into tile t's S columns
        auto issue_s = [&](int t, uint32_t tk) {
          const uint64_t qd = sdesc_adv(q_desc, t * Cfg::Q_BYTES), kd = sdesc_adv(k_desc, (tk & 1u) * Cfg::KV_BYTES);
  #pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            if (leader) umma_f16_ss(tmem + (Cfg::S_COL_STRIDE * t), sdesc_adv(qd, off), sdesc_adv(kd, off), idesc_s,
                                    kk > 0 ? 1u : 0u);
          }
          if (leader) umma_commit(&s_full[t]);
        };
        // Issue order per item: S_A(0) S_B(0) | PV_A(j) S_A(j+1) PV_B(j) S_B(j+1) | ...  tcgen05.mma
        // executes in issue order, so S_t(j+1) may follow PV_t(j), which reads P_t(j) from
        // the same TMEM columns, without waiting for it; each softmax warpgroup then has the
        // other tile's PV and S (1024 tensor-core cycles) to hide behind.  Across items the
        // same holds: the next item's S_A(0), S_B(0) follow the last PV_A, PV_B at once and
        // run while the softmax warps write the item's output; its first PV, which starts O
        // afresh, waits for P, which the warps store only after that output has left TMEM.
        uint32_t tk = 0;            // K/V tiles consumed over all items
        uint32_t ns[2] = {0u, 0u};  // S tiles issued per tile slot over all items (P barrier phases)
        bool ok = true;
        FwdItem x;
        // Per-lane waits (lane_wait) inside an item: a lane whose wait gives up skips the rest of
        // the item's work and meets the others at the item's __syncwarp and the next vote, so
        // every lane runs the same warp collectives.
        for (int ci = 0;; ++ci) {
          const bool got = ok && read_item(ci, x);
          if (!__all_sync(0xffffffffu, got)) break;
          bool iok = lane_wait(q_full, (uint32_t)ci & 1u, abort_flag, kSiteAttnQ) &&
                     lane_wait(&k_full[tk & 1u], (tk >> 1) & 1u, abort_flag, kSiteAttnKFull);
          if (iok) {
            tc_fence_after();
            for (int t = 0; t < 2; ++t)
              if (x.nkv[t] > 0) issue_s(t, tk);
            if (leader) umma_commit(&k_empty[tk & 1u]);
            if (x.n_j == 1 && leader) umma_commit(q_empty);  // the item's last S has read Q
          }
          for (int j = 0; j < x.n_j && iok; ++j) {
            const uint32_t tv = tk + (uint32_t)j, tn = tv + 1u;  // V_j, K_{j+1} ring counts
            bool k_next = false;  // K_{j+1} has landed
            if (!lane_wait(&v_full[tv & 1u], (tv >> 1) & 1u, abort_flag, kSiteAttnVFull)) { iok = false; break; }
            const uint64_t vd = sdesc_adv(v_desc, (tv & 1u) * Cfg::KV_BYTES);
            for (int t = 0; t < 2 && iok; ++t) {
              if (j >= x.nkv[t]) continue;
              // O_t += P_t V_j, P_t from TMEM (K = 128 keys), each 64-key half as soon as it is stored
              for (int hf = 0; hf < 2 && iok; ++hf) {
                if (!lane_wait(&p_full[2 * t + hf], (ns[t] + (uint32_t)j) & 1u, abort_flag, kSiteAttnPFull)) {
                  iok = false;
                  break;
                }
                tc_fence_after();
  #pragma unroll
                for (int k4 = 0; k4 < 4; ++k4) {
                  const int kk = 4 * hf + k4;
                  if (leader) umma_f16_ts(tmem + Cfg::O_COL0 + t * D, tmem + (Cfg::S_COL_STRIDE * t) + kk * 8,
                                          sdesc_adv(vd, kk * 2048), idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
                }
              }
              if (!iok) break;
              if (j == x.nkv[t] - 1 && leader) umma_commit(&o_full[t]);
              if (j + 1 < x.nkv[t]) {
                if (!k_next) {
                  if (!lane_wait(&k_full[tn & 1u], (tn >> 1) & 1u, abort_flag, kSiteAttnKFull)) {
                    iok = false;
                    break;
                  }
                  tc_fence_after();
                  k_next = true;
                }
                issue_s(t, tn);
              }
            }
            if (!iok) break;
            if (leader) umma_commit(&v_empty[tv & 1u]);
            if (k_next && leader) umma_commit(&k_empty[tn & 1u]);
            if (j + 2 == x.n_j && leader) umma_commit(q_empty);  // S(n_j - 1) were the item's last S
          }
          ok = iok;
          tk += (uint32_t)x.n_j;
          ns[0] += (uint32_t)x.nkv[0];
          ns[1] += (uint32_t)x.nkv[1];
          __syncwarp();
          if (ok && leader) mbar_arrive(&item_empty[ci % kFwdItemRing]);
        }
        if (leader) umma_commit(drain);
        volatile int no_abort = 0;
        warp_wait(drain, 0, &no_abort, kSiteAttnDrain);
      }
    }
  } else {
    warpgroup_reg_alloc<216>();
    // ---------------------------------------------------------------- softmax (warps 4-7: A, 8-11: B)
    const int t = (warp < 8) ? 0 : 1;
    const uint32_t quarter = warp & 3u;
    const int r = (int)(quarter * 32 + lane);  // row within the Q tile == TMEM lane
    const uint32_t lane_base = (quarter * 32u) << 16;
    const uint32_t s_col = (Cfg::S_COL_STRIDE * t), o_col = Cfg::O_COL0 + t * D;
    uint32_t ns = 0, no = 0;  // S tiles and outputs of this tile slot over all items (barrier phases)
    bool ok = true;
    for (int ci = 0; ok; ++ci) {
      FwdItem x;
      const bool more = __all_sync(0xffffffffu, read_item(ci, x));
      if (lane == 0) mbar_arrive(&item_empty[ci % kFwdItemRing]);
      if (!more) break;
      const int nkv = x.nkv[t];
      const int qi = x.q0[t] + r;  // query index
      const int bh = x.bh;
      float m_used = -INFINITY, l = 0.0f;
      // RECOMP: the exponent offset of the row, from the saved LSE (rows at or beyond S: -inf)
      const float nl2 = RECOMP ? (qi < p.S ? p.lse_in[(long long)bh * p.S + qi] * -1.4426950408889634f : -INFINITY)
                               : 0.0f;
      for (int j = 0; j < nkv; ++j) {
        // warp-uniform outcome: the tcgen05.ld / st that follow are warp-collective
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[t], (ns + (uint32_t)j) & 1u, abort_flag, kSiteAttnSFull))) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t xu[128];  // the S row, loaded straight into the registers it is used from
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_base + s_col + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&xu[32 * c]));
        tmem_wait_ld();
        float* xs = reinterpret_cast<float*>(xu);
        const int k0 = j * 128;
        int limit = p.S - k0;                           // keys at or beyond S are masked
        if (p.causal) limit = min(limit, qi - k0 + 1);  // keys after the query are masked
        const bool unmasked = __all_sync(0xffffffffu, limit >= 128);
        if (!unmasked) {
#pragma unroll
          for (int c = 0; c < 128; ++c) xs[c] = (c < limit) ? xs[c] : -INFINITY;
        }
        if constexpr (RECOMP) {
          if (unmasked)
            softmax_p_to_tmem<true>(xs, p.scale_log2, nl2, tmem + lane_base + s_col, &p_full[2 * t]);
          else
            softmax_p_to_tmem<false>(xs, p.scale_log2, nl2, tmem + lane_base + s_col, &p_full[2 * t]);
          continue;
        }
        float mx;
        {  // tree reduction: 8 independent chains of three-input maxima
          float m8[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) m8[u] = fmaxf(xs[u], xs[8 + u]);
#pragma unroll
          for (int c = 16; c < 128; c += 16)
#pragma unroll
            for (int u = 0; u < 8; ++u) m8[u] = fmax3(m8[u], xs[c + u], xs[c + 8 + u]);
          mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
        }
        mx *= p.scale_log2;
        const float m_new = fmaxf(m_used, mx);
        if (j == 0) {
          m_used = m_new;
        } else {
          const bool need = m_new > m_used + 8.0f;
          if (__any_sync(0xffffffffu, need)) {
            // O_t holds PV(j-1) (S_t(j) was issued after it completed); no PV is in flight
            const float alpha = need ? ex2_approx(m_used - m_new) : 1.0f;
            if (need) {
              l *= alpha;
              m_used = m_new;
            }
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
              uint32_t u[32];
              tmem_ld32(tmem + lane_base + o_col + c * 32, u);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * alpha);
              tmem_st32(tmem + lane_base + o_col + c * 32, u);
            }
          }
        }
        // P = exp2(x * scale_log2 - m_used) -> bf16 pairs into TMEM columns [s_col, s_col + 64)
        if (unmasked)
          l += softmax_p_to_tmem<true>(xs, p.scale_log2, -m_used, tmem + lane_base + s_col, &p_full[2 * t]);
        else
          l += softmax_p_to_tmem<false>(xs, p.scale_log2, -m_used, tmem + lane_base + s_col, &p_full[2 * t]);
      }
      if (!ok) break;
      ns += (uint32_t)nkv;
      if (nkv == 0) continue;  // a second tile beyond S: nothing computed, nothing stored
      // the item's output leaves TMEM before these warps store the next item's first P,
      // which is what the next item's first PV (overwriting O_t) waits for
      if (!__all_sync(0xffffffffu, mbar_wait(&o_full[t], no & 1u, abort_flag, kSiteAttnOFull))) {
        ok = false;
        break;
      }
      ++no;
      tc_fence_after();
      if constexpr (RECOMP) {
        // epilogue: Dt = rowsum(dO * O) and lse2 for the backward
        const bool row_ok = qi < p.S;
        const uint4* drow = reinterpret_cast<const uint4*>(p.dout + ((long long)bh * p.S + (row_ok ? qi : 0)) * D);
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint4 dv4[4] = {};
          if (row_ok) {
#pragma unroll
            for (int i = 0; i < 4; ++i) dv4[i] = __ldg(drow + c * 4 + i);
          }
          uint32_t u[32];
          tmem_ld32(tmem + lane_base + o_col + c * 32, u);  // warp-collective: every lane
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&dv4[i]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 d2 = __bfloat1622float2(h2[e]);
              acc[i] = fmaf(__uint_as_float(u[8 * i + 2 * e]), d2.x, acc[i]);
              acc[i] = fmaf(__uint_as_float(u[8 * i + 2 * e + 1]), d2.y, acc[i]);
            }
          }
        }
        if (qi < p.S_pad) {  // rows of a query tile past the last one do not exist in Dt / lse2
          const long long rr = (long long)bh * p.S_pad + qi;
          p.dt[rr] = row_ok ? (acc[0] + acc[1]) + (acc[2] + acc[3]) : 0.0f;
          p.lse2[rr] = row_ok ? nl2 : -INFINITY;
        }
      } else {
        // epilogue: O / l -> bf16, LSE
        const float inv = 1.0f / l;
        const bool out32 = (reinterpret_cast<uintptr_t>(p.out) & 31u) == 0;
        const int b = bh / p.Hq, h = bh % p.Hq;
        __nv_bfloat16* orow = p.out + (p.out_tokens ? (((long long)b * p.S + qi) * p.Hq + h) * D
                                                    : ((long long)bh * p.S + qi) * D);
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t u[32];
          tmem_ld32(tmem + lane_base + o_col + c * 32, u);
          tmem_wait_ld();
          if (qi < p.S) {  // 32-byte stores where `out` allows: each fills a whole sector of the row
#pragma unroll
            for (int e = 0; e < 32; e += 16) {
              uint32_t wv[8];
#pragma unroll
              for (int i = 0; i < 8; ++i)
                wv[i] = pack_bf16x2(__uint_as_float(u[e + 2 * i]) * inv, __uint_as_float(u[e + 2 * i + 1]) * inv);
              if (out32) {
                stg256(orow + c * 32 + e, wv[0], wv[1], wv[2], wv[3], wv[4], wv[5], wv[6], wv[7]);
              } else {  // out only 16-byte aligned
                *reinterpret_cast<uint4*>(orow + c * 32 + e) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
                *reinterpret_cast<uint4*>(orow + c * 32 + e + 8) = make_uint4(wv[4], wv[5], wv[6], wv[7]);
              }
            }
          }
        }
        if (qi < p.S) p.lse[(long long)bh * p.S + qi] = (m_used + __log2f(l)) * 0.69314718055994531f;
      }
      tc_fence_before();
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

// ---------------------------------------------------------------------------
// Exact SIMT attention (fp32 FFMA, accurate expf/logf): the f32 path and any
// head_dim the tensor-core kernels do not cover.  One thread per query row
// (forward, dQ) or key row (dK/dV); K/V (or Q/dO) rows staged through shared memory.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float ldx(const T* p);
template <>
__device__ __forceinline__ float ldx<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ldx<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <typename T>
__device__ __forceinline__ void stx(T* p, float v);
template <>
__device__ __forceinline__ void stx<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void stx<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

constexpr int kSimtRows = 64;   // rows per CTA (one per thread)
constexpr int kSimtTile = 32;   // staged rows per step
constexpr int kSimtMaxD = 128;

// grid: (ceil(S/64), B*Hq); block 64.  scale: natural-units softmax scale.
template <typename T, int D>
__global__ void __launch_bounds__(kSimtRows) k_attn_fwd_simt(T* __restrict__ out, float* __restrict__ lse,
                                                             const T* __restrict__ q, const T* __restrict__ k,
                                                             const T* __restrict__ v, int Hq, int Hkv, int S,
                                                             int causal, float scale) {
  __shared__ float ks[kSimtTile][D + 1];
  __shared__ float vs[kSimtTile][D + 1];
  const int bh = blockIdx.y, b = bh / Hq, h = bh % Hq;
  const long long kvh = (long long)b * Hkv + h / (Hq / Hkv);
  const int i = blockIdx.x * kSimtRows + threadIdx.x;
  float qr[D], o[D];
  const T* qp = q + ((long long)bh * S + (i < S ? i : 0)) * D;
#pragma unroll
  for (int d = 0; d < D; ++d) {
    qr[d] = ldx(qp + d);
    o[d] = 0.0f;
  }
  float m = -INFINITY, l = 0.0f;
  const int row_last = min(S, (int)(blockIdx.x + 1) * kSimtRows) - 1;
  const int jend = causal ? row_last + 1 : S;
  for (int j0 = 0; j0 < jend; j0 += kSimtTile) {
    __syncthreads();
    for (int e = threadIdx.x; e < kSimtTile * D; e += kSimtRows) {
      const int jj = e / D, d = e % D;
      const int j = j0 + jj;
      ks[jj][d] = j < S ? ldx(k + (kvh * S + j) * D + d) : 0.0f;
      vs[jj][d] = j < S ? ldx(v + (kvh * S + j) * D + d) : 0.0f;
    }
    __syncthreads();
    if (i < S) {
      for (int jj = 0; jj < kSimtTile; ++jj) {
        const int j = j0 + jj;
        if (j >= S || (causal && j > i)) break;
        float s = 0.0f;
#pragma unroll
        for (int d = 0; d < D; ++d) s = fmaf(qr[d], ks[jj][d], s);
        s *= scale;
        const float mn = fmaxf(m, s);
        const float a = expf(m - mn), pj = expf(s - mn);
        l = l * a + pj;
#pragma unroll
        for (int d = 0; d < D; ++d) o[d] = fmaf(pj, vs[jj][d], o[d] * a);
        m = mn;
      }
    }
  }
  if (i < S) {
    T* op = out + ((long long)bh * S + i) * D;
#pragma unroll
    for (int d = 0; d < D; ++d) stx(op + d, o[d] / l);
    lse[(long long)bh * S + i] = m + logf(l);
  }
}

// dQ and the row term Dt[i] = sum_j P_ij dP_ij.  grid (ceil(S/64), B*Hq), block 64.
template <typename T, int D>
__global__ void __launch_bounds__(kSimtRows) k_attn_bwd_dq_simt(T* __restrict__ dq, float* __restrict__ dterm,
                                                                const T* __restrict__ dout, const T* __restrict__ q,
                                                                const T* __restrict__ k, const T* __restrict__ v,
                                                                const float* __restrict__ lse, int Hq, int Hkv, int S,
                                                                int causal, float scale) {
  __shared__ float ks[kSimtTile][D + 1];
  __shared__ float vs[kSimtTile][D + 1];
  const int bh = blockIdx.y, b = bh / Hq, h = bh % Hq;
  const long long kvh = (long long)b * Hkv + h / (Hq / Hkv);
  const int i = blockIdx.x * kSimtRows + threadIdx.x;
  const int ic = i < S ? i : 0;
  float qr[D], dor[D], acc[D];
#pragma unroll
  for (int d = 0; d < D; ++d) {
    qr[d] = ldx(q + ((long long)bh * S + ic) * D + d);
    dor[d] = ldx(dout + ((long long)bh * S + ic) * D + d);
    acc[d] = 0.0f;
  }
  const float L = lse[(long long)bh * S + ic];
  const int row_last = min(S, (int)(blockIdx.x + 1) * kSimtRows) - 1;
  const int jend = causal ? row_last + 1 : S;
  float dt = 0.0f;
  // pass 1: Dt = sum_j P dP ; pass 2: dQ = scale sum_j P (dP - Dt) K_j
  for (int pass = 0; pass < 2; ++pass) {
    for (int j0 = 0; j0 < jend; j0 += kSimtTile) {
      __syncthreads();
      for (int e = threadIdx.x; e < kSimtTile * D; e += kSimtRows) {
        const int jj = e / D, d = e % D;
        const int j = j0 + jj;
        ks[jj][d] = j < S ? ldx(k + (kvh * S + j) * D + d) : 0.0f;
        vs[jj][d] = j < S ? ldx(v + (kvh * S + j) * D + d) : 0.0f;
      }
      __syncthreads();
      if (i < S) {
        for (int jj = 0; jj < kSimtTile; ++jj) {
          const int j = j0 + jj;
          if (j >= S || (causal && j > i)) break;
          float s = 0.0f, dp = 0.0f;
#pragma unroll
          for (int d = 0; d < D; ++d) {
            s = fmaf(qr[d], ks[jj][d], s);
            dp = fmaf(dor[d], vs[jj][d], dp);
          }
          const float pj = expf(s * scale - L);
          if (pass == 0) {
            dt = fmaf(pj, dp, dt);
          } else {
            const float ds = pj * (dp - dt);
#pragma unroll
            for (int d = 0; d < D; ++d) acc[d] = fmaf(ds, ks[jj][d], acc[d]);
          }
        }
      }
    }
  }
  if (i < S) {
#pragma unroll
    for (int d = 0; d < D; ++d) stx(dq + ((long long)bh * S + i) * D + d, acc[d] * scale);
    dterm[(long long)bh * S + i] = dt;
  }
}

// dK, dV for one key row per thread, summed over the query heads of its KV group.
// grid (ceil(S/64), B*Hkv), block 64.
template <typename T, int D>
__global__ void __launch_bounds__(kSimtRows) k_attn_bwd_dkv_simt(T* __restrict__ dk, T* __restrict__ dv,
                                                                 const T* __restrict__ dout, const T* __restrict__ q,
                                                                 const T* __restrict__ k, const T* __restrict__ v,
                                                                 const float* __restrict__ lse,
                                                                 const float* __restrict__ dterm, int Hq, int Hkv,
                                                                 int S, int causal, float scale) {
  __shared__ float qs[kSimtTile][D + 1];
  __shared__ float dos[kSimtTile][D + 1];
  __shared__ float ls[kSimtTile], dts[kSimtTile];
  const int kvbh = blockIdx.y, b = kvbh / Hkv, hk = kvbh % Hkv;
  const int group = Hq / Hkv;
  const int j = blockIdx.x * kSimtRows + threadIdx.x;
  const int jc = j < S ? j : 0;
  float kr[D], vr[D], dka[D], dva[D];
#pragma unroll
  for (int d = 0; d < D; ++d) {
    kr[d] = ldx(k + ((long long)kvbh * S + jc) * D + d);
    vr[d] = ldx(v + ((long long)kvbh * S + jc) * D + d);
    dka[d] = 0.0f;
    dva[d] = 0.0f;
  }
  const int istart = causal ? (int)blockIdx.x * kSimtRows : 0;
  for (int g = 0; g < group; ++g) {
    const long long bh = (long long)b * Hq + hk * group + g;
    for (int i0 = istart; i0 < S; i0 += kSimtTile) {
      __syncthreads();
      for (int e = threadIdx.x; e < kSimtTile * D; e += kSimtRows) {
        const int ii = e / D, d = e % D;
        const int i = i0 + ii;
        qs[ii][d] = i < S ? ldx(q + (bh * S + i) * D + d) : 0.0f;
        dos[ii][d] = i < S ? ldx(dout + (bh * S + i) * D + d) : 0.0f;
      }
      for (int ii = threadIdx.x; ii < kSimtTile; ii += kSimtRows) {
        const int i = i0 + ii;
        ls[ii] = i < S ? lse[bh * S + i] : 0.0f;
        dts[ii] = i < S ? dterm[bh * S + i] : 0.0f;
      }
      __syncthreads();
      if (j < S) {
        for (int ii = 0; ii < kSimtTile; ++ii) {
          const int i = i0 + ii;
          if (i >= S) break;
          if (causal && i < j) continue;
          float s = 0.0f, dp = 0.0f;
#pragma unroll
          for (int d = 0; d < D; ++d) {
            s = fmaf(qs[ii][d], kr[d], s);
            dp = fmaf(dos[ii][d], vr[d], dp);
          }
          const float pij = expf(s * scale - ls[ii]);
          const float ds = pij * (dp - dts[ii]);
#pragma unroll
          for (int d = 0; d < D; ++d) {
            dva[d] = fmaf(pij, dos[ii][d], dva[d]);
            dka[d] = fmaf(ds, qs[ii][d], dka[d]);
          }
        }
      }
    }
  }
  if (j < S) {
#pragma unroll
    for (int d = 0; d < D; ++d) {
      stx(dk + ((long long)kvbh * S + j) * D + d, dka[d] * scale);
      stx(dv + ((long long)kvbh * S + j) * D + d, dva[d]);
    }
  }
}

}  // namespace beacon
