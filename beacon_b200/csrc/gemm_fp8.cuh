// gemm_fp8.cuh -- GEMM with fp8 e4m3 weights decoded inside the pipeline.
//
// out[M,N] = (A[M,K] . decode(W[K,N])) * scale (+ bias), A bf16 K-major, W fp8 e4m3 row-major
// ([K][N], N contiguous: the MN-major B operand), fp32 accumulation, bf16 out.  Each weight
// byte crosses HBM once: TMA brings the raw fp8 tile into a staging buffer, converter warps
// decode it to bf16 straight into the 128-byte swizzled operand layout the MMA reads, and
// the bf16 tensor cores multiply.  (Decoding to a bf16 copy in HBM first would move 1 B in,
// 2 B out and 2 B back per weight element, plus a launch.)
//
// A 2-CTA cluster computes a 256x256 tile with tcgen05.mma.cta_group::2 (M = 256 over the
// pair): each CTA TMA-loads its own 128 rows of A and the fp8 bytes of its own 128-column
// half of W, and its converter warps decode that half (128 x 64 values per 64-deep K step).
// No load uses cluster multicast.
//
//   warp 0      TMA producer (both CTAs): A pair loads complete on the leader's `full`
//               barrier, the fp8 staging tile on this CTA's `stg_full`.
//   warp 1      (leader) MMA issuer: the whole warp runs the loop, one elected lane issues.
//   warps 2-5   epilogue (both CTAs), as in the bf16 GEMM.
//   warps 6-15  converters (both CTAs), one group of two warps per stage: wait stg_full,
//               decode, fence the generic-proxy stores for the tensor core, arrive on the
//               leader's `full` barrier.
// The leader's full[s] completes when both CTAs' A bytes have landed and stage s's converter
// warps of both CTAs have stored their B halves; the MMAs' commit to both CTAs' empty[s]
// then frees A, B and the staging buffer of stage s for the next round.
//
// Measured on B200 (4096^3), with HBM reads of 1 byte per weight element: 0.35 ms with one
// set of converter warps decoding item by item; 0.27 ms with loads, decodes and stores
// batched per thread and eight warps; about 0.15 ms with every stage decoded at once by its
// own group (a timestamp trace had shown the converters busy back to back at 0.7-0.9 us
// per K step against 0.26 us of MMA, most of it the stores, fence and arrive of a stage).
//
// Decoding (restating F8E4M3::to_f32, crates/beacon-core/src/dtype.rs:138-161, without the
// per-element branches): the byte's 7 exponent-mantissa bits are placed in a bf16 at bit 4
// (exponent field e, mantissa m << 4) and the sign at bit 15; that bf16 is 2^-120 times the
// e4m3 value for every finite code, subnormals included (bf16 subnormals are multiples of
// 2^-133 and e4m3 subnormals of 2^-9), so one exact bf16x2 multiply by 2^120 finishes two
// values.  The e4m3 NaN codes (0x7f, 0xff) would come out as 480; their exponent field is
// then forced to all ones.
#pragma once

#include "gemm.cuh"
#include "sm100.cuh"

namespace beacon {

struct GemmFp8Cfg {
  static constexpr int BM = 128, BN = 256, BK = 64, STAGES = 5;
  static constexpr uint32_t A_BYTES = BM * BK * 2;         // this CTA's 128 rows of A (bf16)
  static constexpr uint32_t B_BYTES = (BN / 2) * BK * 2;   // this CTA's decoded half of W (bf16)
  static constexpr uint32_t STG_BYTES = (BN / 2) * BK;     // the same half as fp8 bytes
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr size_t SMEM_BYTES =
      1024 + (size_t)STAGES * (A_BYTES + B_BYTES + STG_BYTES) + 256;
  static constexpr int CONV_WARP0 = 6;
  // The converter warps form one group per stage; group g decodes stage g's K steps (g,
  // g + STAGES, ...), so all stages are decoded at once: a stage's decode is short, but its
  // stores, the proxy fence and the cluster-scope arrive that hands it to the MMA take far
  // longer, and converters working through the stages one after another bounded the kernel
  // (0.26 ms at 4096^3 against 0.16 with four stages decoding at once).  A group owning its
  // stage waits on that stage's barrier phases strictly in order: groups taking K steps in
  // turn over more stages than groups could wait on a phase two ahead of the barrier's, which
  // a parity wait cannot tell from the phase before.
  static constexpr int GROUP_WARPS = 2;
  static constexpr int CONV_GROUPS = STAGES;
  static constexpr int CONV_WARPS = CONV_GROUPS * GROUP_WARPS;
  static constexpr int THREADS = (CONV_WARP0 + CONV_WARPS) * 32;
  static constexpr int ITEMS = 1024 / (GROUP_WARPS * 32);  // (K row, 8-column chunk) items per thread
  static_assert(ITEMS % 8 == 0, "8-item batches");
};

enum : unsigned int {
  kSiteFp8Stg = 0x121,
  kSiteFp8Drain = 0x122,
};

// Two e4m3 bytes, spread one per 16-bit half (byte in bits 0-7), to a bf16x2 word.
__device__ __forceinline__ uint32_t e4m3x2_to_bf16x2(uint32_t x) {
  const uint32_t em = x & 0x007f007fu;
  const uint32_t bits = (em << 4) | ((x << 8) & 0x80008000u);
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(bits), "r"(0x7B807B80u));  // x 2^120 (exact)
  const uint32_t n7 = (em + 0x00010001u) & 0x00800080u;  // 0x80 in each half where em == 0x7f (NaN)
  return r | (n7 * 0xffu);                                // exponent field all ones: 480 -> NaN
}

// Eight e4m3 bytes (a uint2) to eight bf16 values (a uint4), element order preserved.
__device__ __forceinline__ uint4 e4m3x8_to_bf16x8(uint2 w) {
  uint4 o;
  o.x = e4m3x2_to_bf16x2(__byte_perm(w.x, 0u, 0x4140));
  o.y = e4m3x2_to_bf16x2(__byte_perm(w.x, 0u, 0x4342));
  o.z = e4m3x2_to_bf16x2(__byte_perm(w.y, 0u, 0x4140));
  o.w = e4m3x2_to_bf16x2(__byte_perm(w.y, 0u, 0x4342));
  return o;
}

__global__ void __launch_bounds__(GemmFp8Cfg::THREADS, 1)
    k_gemm_fp8w_tc2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                    const GemmParams p) {
  using Cfg = GemmFp8Cfg;
  constexpr int BK = Cfg::BK, STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * Cfg::A_BYTES;
  uint8_t* sStg = sB + STAGES * Cfg::B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sStg + STAGES * Cfg::STG_BYTES);  // used in the leader
  uint64_t* empty = full + STAGES;
  uint64_t* stg_full = empty + STAGES;
  uint64_t* tfull = stg_full + STAGES;  // [2]
  uint64_t* tempty = tfull + 2;         // [2] used in the leader: 4 epilogue warps x 2 CTAs
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = (int)(blockIdx.x >> 1), n_clusters = (int)(gridDim.x >> 1);
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1 + 2 * Cfg::GROUP_WARPS);  // the leader's expect_tx arrive + a group's warps x 2 CTAs
      mbar_init(&empty[s], 1);
      mbar_init(&stg_full[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrive or commit
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.tiles_m * p.tiles_n;  // tiles of 256 x 256
  const int ktiles = (p.K + BK - 1) / BK;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, issued_parity = 0;
      bool ok = true;
      for (int tile = cluster; tile < num_tiles && ok; tile += n_clusters) {
        const int tm = tile / p.tiles_n, tn = tile % p.tiles_n;
        const int m0 = tm * 256 + 128 * (int)rank;
        const int n0 = tn * 256 + 128 * (int)rank;
        for (int kt = 0; kt < ktiles; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteGemmEmpty)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::A_BYTES);
          const int k0 = kt * BK;
          tma_load_2d_pair(sA + stage * Cfg::A_BYTES, &tmA, cluster_map(&full[stage], 0), k0, m0);
          mbar_arrive_expect_tx(&stg_full[stage], Cfg::STG_BYTES);
          tma_load_2d(sStg + stage * Cfg::STG_BYTES, &tmW, &stg_full[stage], n0, k0);
          issued |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // every copy in flight must land before the CTA exits: this CTA's staging loads on
        // its own barriers, and (leader) both CTAs' A loads on the leader's
        volatile int no_abort = 0;
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) {
            mbar_wait(&stg_full[s], (issued_parity >> s) & 1u, &no_abort, kSiteFp8Drain);
            if (leader) mbar_wait(&full[s], (issued_parity >> s) & 1u, &no_abort, kSiteFp8Drain);
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA only)
    if (leader) {
      const bool issuer = elect_one();
      constexpr uint32_t idesc = make_idesc_f16(256, Cfg::BN, false, true);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = cluster; tile < num_tiles && ok; tile += n_clusters) {
        if (!warp_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, kSiteGemmTmemEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * Cfg::BN);
        for (int kt = 0; kt < ktiles; ++kt) {
          // cluster-scope acquire: the peer's converters stored half of B with generic stores
          if (!warp_wait_cluster(&full[stage], phase, abort_flag, kSiteGemmFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = make_sdesc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = make_sdesc_sw128(b_addr + kk * 2048, 64 * BK * 2, 1024);
            if (issuer) umma_f16_ss_pair(d, ad, bd, idesc, (kt | kk) != 0 ? 1u : 0u);
          }
          if (issuer) umma_commit_pair(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (issuer) umma_commit_pair(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (issuer) umma_commit_leader(drain);
      volatile int no_abort = 0;
      warp_wait(drain, 0, &no_abort, kSiteGemmDrain);
    }
  } else if (warp < Cfg::CONV_WARP0) {
    // ------------------------------------------------------------ epilogue (warps 2..5, both CTAs)
    const uint32_t q = warp & 3u;
    const uint32_t tempty_leader[2] = {cluster_map(&tempty[0], 0), cluster_map(&tempty[1], 0)};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = cluster; tile < num_tiles; tile += n_clusters) {
      const int tm = tile / p.tiles_n, tn = tile % p.tiles_n;
      const bool got = mbar_wait(&tfull[acc], acc_phase, abort_flag, kSiteGemmTmemFull);
      if (!__all_sync(0xffffffffu, got)) break;  // warp-uniform: tcgen05.ld below is warp-collective
      tc_fence_after();
      const int row = tm * 256 + 128 * (int)rank + (int)(q * 32 + lane);
      gemm_epilogue_tile<Cfg::BN>(p, row, tmem_base + ((q * 32u) << 16) + (uint32_t)(acc * Cfg::BN), tn, false);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  } else {
    // ------------------------------------------------------------ converters (warps 6.., both CTAs)
    // Group g decodes stage g: K steps g, g + STAGES, ... of the CTA's whole sequence (all tiles).
    // Item (k, c): K row k (0..63) and 8-column chunk c (0..15) of this CTA's 128 columns.
    // Thread ct of a group takes items ct + NCT j: a warp reads two whole 128-byte staging
    // rows and writes four whole 128-byte rows of the swizzled bf16 operand (no bank
    // conflicts).
    constexpr int NCT = Cfg::GROUP_WARPS * 32;
    const int cw = (int)warp - Cfg::CONV_WARP0;
    const int grp = cw / Cfg::GROUP_WARPS;
    const int ct = (cw % Cfg::GROUP_WARPS) * 32 + (int)lane;
    const int n_steps = ((num_tiles - cluster + n_clusters - 1) / n_clusters) * ktiles;  // this cluster's K steps
    const int stage = grp;
    uint32_t phase = 0;
    for (int step = grp; step < n_steps; step += STAGES, phase ^= 1u) {
      if (!__all_sync(0xffffffffu, mbar_wait(&stg_full[stage], phase, abort_flag, kSiteFp8Stg))) break;
      // loads, decodes and stores in batches of eight: the items are independent, so their
      // latencies overlap (decoded one after another, a stage took ~4x longer)
      const uint32_t stg = smem_u32(sStg + stage * Cfg::STG_BYTES);
      const uint32_t b = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
      for (int j0 = 0; j0 < Cfg::ITEMS; j0 += 8) {
        uint2 w[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int it = ct + NCT * (j0 + j);
          const int k = it >> 4, c = it & 15;
          asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(w[j].x), "=r"(w[j].y) : "r"(stg + k * 128 + c * 8)
                       : "memory");
        }
        uint4 o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = e4m3x8_to_bf16x8(w[j]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int it = ct + NCT * (j0 + j);
          const int k = it >> 4, c = it & 15;
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(b + (c >> 3) * 8192 + k * 128 +
                                                                        (((c & 7) ^ (k & 7)) << 4)),
                       "r"(o[j].x), "r"(o[j].y), "r"(o[j].z), "r"(o[j].w)
                       : "memory");
        }
      }
      fence_proxy_async_smem();  // generic-proxy stores -> the tensor core's async proxy
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cluster_map(&full[stage], 0));
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still arrive on its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace beacon
