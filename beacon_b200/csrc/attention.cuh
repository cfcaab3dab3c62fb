// attention.cuh -- causal scaled-dot-product attention on tcgen05 tensor cores.
//
// Forward (kernel ID `attention_adjoint_fwd`, crates/beacon-cuda/src/attention.rs:21-40):
// one CTA per (query tile of 128 rows, batch*head); online softmax in the log2
// domain with fp32 statistics; LSE written in natural-log units.
//
//   warp 0     TMA producer: Q once, then K_j and V_j (128 keys x D) into 2-deep rings.
//   warp 1     TMEM allocator + tcgen05.mma issuer:
//                S[j&1] = Q K_j^T        (M=128, N=128, K=D;   A,B K-major in smem)
//                O     += P[j&1] V_j     (M=128, N=D,   K=128; P K-major, V MN-major)
//              S_{j+1} is issued before O += P_j V_j so the tensor core works on
//              the next scores while the softmax warps turn S_j into P_j.
//   warps 2-5  softmax: one query row per thread (TMEM lane = row), P_j written
//              to shared memory as bf16 in the 128B-swizzled K-major layout the
//              MMA reads.  O is rescaled in TMEM only when a row maximum grows by
//              more than 2^8 (the final O / l is exact either way because P and l
//              use the same stale maximum); then the epilogue normalises O.
//
// TMEM: S0 cols [0,128), S1 [128,256), O [256, 256+D).
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
};

template <int D>
struct AttnFwdCfg {
  static constexpr int BM = 128, BN = 128;
  static constexpr uint32_t Q_BYTES = BM * D * 2;
  static constexpr uint32_t KV_BYTES = BN * D * 2;
  static constexpr uint32_t P_BYTES = BM * BN * 2;
  static constexpr size_t SMEM_BYTES = 1024 + Q_BYTES + 4 * (size_t)KV_BYTES + 2 * (size_t)P_BYTES + 512;
  static constexpr int THREADS = 192;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t O_COL = 256;
};

enum : unsigned int {
  kSiteAttnQ = 0x201,
  kSiteAttnKFull = 0x202,
  kSiteAttnKEmpty = 0x203,
  kSiteAttnVFull = 0x204,
  kSiteAttnVEmpty = 0x205,
  kSiteAttnSFull = 0x206,
  kSiteAttnSFree = 0x207,
  kSiteAttnPFull = 0x208,
  kSiteAttnPEmpty = 0x209,
  kSiteAttnOFull = 0x20a,
  kSiteAttnDrain = 0x20b,
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Loads one 128-row x D tile (rows `row0..row0+127` of head `z`) as D/64 swizzled
// column blocks of 128 rows x 128 bytes.
template <int D>
__device__ __forceinline__ void tma_load_rows(uint8_t* dst, const CUtensorMap* m, uint64_t* bar, int row0, int z) {
#pragma unroll
  for (int b = 0; b < D / 64; ++b) tma_load_3d(dst + b * 128 * 128, m, bar, b * 64, row0, z);
}

template <int D>
__global__ void __launch_bounds__(192, 1)
    k_attn_fwd_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using Cfg = AttnFwdCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Cfg::Q_BYTES;             // [2]
  uint8_t* sV = sK + 2 * Cfg::KV_BYTES;        // [2]
  uint8_t* sP = sV + 2 * Cfg::KV_BYTES;        // [2]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * Cfg::P_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* s_free = bars + 11;  // [2]
  uint64_t* p_full = bars + 13;  // [2]
  uint64_t* p_empty = bars + 15; // [2]
  uint64_t* o_full = bars + 17;
  uint64_t* drain = bars + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id(), lane = lane_id();
  const int n_bh = p.B * p.Hq;
  const int qt = p.n_qtiles - 1 - (int)(blockIdx.x / n_bh);  // heaviest causal tiles first
  const int bh = (int)(blockIdx.x % n_bh);
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int kvz = b * p.Hkv + h / (p.Hq / p.Hkv);
  const int q0 = qt * Cfg::BM;
  const int n_kv = p.causal ? min(qt + 1, (p.S + Cfg::BN - 1) / Cfg::BN) : (p.S + Cfg::BN - 1) / Cfg::BN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_empty[i], 1);
    }
    mbar_init(o_full, 1);
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
      mbar_arrive_expect_tx(q_full, Cfg::Q_BYTES);
      tma_load_rows<D>(sQ, &tmQ, q_full, q0, bh);
      uint32_t kissued = 0, vissued = 0, kpar = 0, vpar = 0;
      bool ok = true;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&k_empty[st], ph ^ 1u, abort_flag, kSiteAttnKEmpty)) { ok = false; break; }
        mbar_arrive_expect_tx(&k_full[st], Cfg::KV_BYTES);
        tma_load_rows<D>(sK + st * Cfg::KV_BYTES, &tmK, &k_full[st], j * Cfg::BN, kvz);
        kissued |= 1u << st;
        kpar = (kpar & ~(1u << st)) | (ph << st);
        if (!mbar_wait(&v_empty[st], ph ^ 1u, abort_flag, kSiteAttnVEmpty)) { ok = false; break; }
        mbar_arrive_expect_tx(&v_full[st], Cfg::KV_BYTES);
        tma_load_rows<D>(sV + st * Cfg::KV_BYTES, &tmV, &v_full[st], j * Cfg::BN, kvz);
        vissued |= 1u << st;
        vpar = (vpar & ~(1u << st)) | (ph << st);
      }
      if (!ok) {
        volatile int no_abort = 0;
        mbar_wait(q_full, 0, &no_abort, kSiteAttnDrain);
        for (int s = 0; s < 2; ++s) {
          if (kissued & (1u << s)) mbar_wait(&k_full[s], (kpar >> s) & 1u, &no_abort, kSiteAttnDrain);
          if (vissued & (1u << s)) mbar_wait(&v_full[s], (vpar >> s) & 1u, &no_abort, kSiteAttnDrain);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_f16(128, 128, false, false);
      constexpr uint32_t idesc_o = make_idesc_f16(128, D, false, true);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, abort_flag, kSiteAttnQ);
      auto issue_pv = [&](int t) -> bool {
        const int st = t & 1;
        const uint32_t ph = (t >> 1) & 1;
        if (!mbar_wait(&p_full[st], ph, abort_flag, kSiteAttnPFull)) return false;
        if (!mbar_wait(&v_full[st], ph, abort_flag, kSiteAttnVFull)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sP + st * Cfg::P_BYTES);
        const uint32_t v_addr = smem_u32(sV + st * Cfg::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < 128 / 16; ++kk) {
          const uint64_t ad = make_sdesc_sw128(p_addr + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = make_sdesc_sw128(v_addr + kk * 2048, 128 * 128, 1024);
          umma_f16_ss(tmem + Cfg::O_COL, ad, bd, idesc_o, (t > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&p_empty[st]);
        umma_commit(&v_empty[st]);
        return true;
      };
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&k_full[st], ph, abort_flag, kSiteAttnKFull)) { ok = false; break; }
        if (!mbar_wait(&s_free[st], ph ^ 1u, abort_flag, kSiteAttnSFree)) { ok = false; break; }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * Cfg::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          const uint64_t ad = make_sdesc_sw128(q_addr + off, 16, 1024);
          const uint64_t bd = make_sdesc_sw128(k_addr + off, 16, 1024);
          umma_f16_ss(tmem + st * 128, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[st]);
        umma_commit(&k_empty[st]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok && n_kv > 0) ok = issue_pv(n_kv - 1);
      if (ok) umma_commit(o_full);
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, kSiteAttnDrain);
    }
  } else {
    // ---------------------------------------------------------------- softmax (warps 2..5)
    const uint32_t quarter = warp & 3u;
    const int r = (int)(quarter * 32 + lane);  // row within the Q tile == TMEM lane
    const int qi = q0 + r;                     // query index
    const uint32_t lane_base = (quarter * 32u) << 16;
    float m_used = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      // warp-uniform outcome: the tcgen05.ld / st that follow are warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[st], ph, abort_flag, kSiteAttnSFull))) { ok = false; break; }
      tc_fence_after();
      float x[128];
      {
        uint32_t u[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          tmem_ld32(tmem + lane_base + st * 128 + c * 32, u);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) x[c * 32 + e] = __uint_as_float(u[e]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[st]);
      // scale + mask, row max
      const int k0 = j * 128;
      int limit = p.S - k0;                         // keys at or beyond S are masked
      if (p.causal) limit = min(limit, qi - k0 + 1);  // keys after the query are masked
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        x[c] = (c < limit) ? x[c] * p.scale_log2 : -INFINITY;
        mx = fmaxf(mx, x[c]);
      }
      // P buffer st must be free (PV_{j-2} done)
      if (!__all_sync(0xffffffffu, mbar_wait(&p_empty[st], ph ^ 1u, abort_flag, kSiteAttnPEmpty))) { ok = false; break; }
      const float m_new = fmaxf(m_used, mx);
      if (j == 0) {
        m_used = m_new;
      } else {
        const bool need = m_new > m_used + 8.0f;
        if (__any_sync(0xffffffffu, need)) {
          // O must hold PV_{j-1} before it is rescaled
          const int pt = (j - 1) & 1;
          if (!__all_sync(0xffffffffu, mbar_wait(&p_empty[pt], ((j - 1) >> 1) & 1, abort_flag, kSiteAttnPEmpty))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float alpha = need ? ex2_approx(m_used - m_new) : 1.0f;
          if (need) {
            l *= alpha;
            m_used = m_new;
          }
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t u[32];
            tmem_ld32(tmem + lane_base + Cfg::O_COL + c * 32, u);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * alpha);
            tmem_st32(tmem + lane_base + Cfg::O_COL + c * 32, u);
          }
          tmem_wait_st();
        }
      }
      // P = exp2(x - m_used) -> bf16, 128B-swizzled K-major rows in sP[st]
      uint8_t* prow = sP + st * Cfg::P_BYTES;
      float lsum = 0.0f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {  // 16 chunks of 8 keys
        float pv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          pv[e] = ex2_approx(x[c * 8 + e] - m_used);
          lsum += pv[e];
        }
        uint4 w;
        w.x = pack_bf16x2(pv[0], pv[1]);
        w.y = pack_bf16x2(pv[2], pv[3]);
        w.z = pack_bf16x2(pv[4], pv[5]);
        w.w = pack_bf16x2(pv[6], pv[7]);
        *reinterpret_cast<uint4*>(prow + (c >> 3) * 16384 + sw128_offset((uint32_t)r, (uint32_t)(c & 7))) = w;
      }
      l += lsum;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[st]);
    }
    // epilogue: O / l -> bf16, LSE
    if (ok && __all_sync(0xffffffffu, mbar_wait(o_full, 0, abort_flag, kSiteAttnOFull))) {
      tc_fence_after();
      const float inv = 1.0f / l;
      __nv_bfloat16* orow = p.out + ((long long)bh * p.S + qi) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t u[32];
        tmem_ld32(tmem + lane_base + Cfg::O_COL + c * 32, u);
        tmem_wait_ld();
        if (qi < p.S) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(u[e + 0]) * inv, __uint_as_float(u[e + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(u[e + 2]) * inv, __uint_as_float(u[e + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(u[e + 4]) * inv, __uint_as_float(u[e + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(u[e + 6]) * inv, __uint_as_float(u[e + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + e) = w;
          }
        }
      }
      if (qi < p.S) p.lse[(long long)bh * p.S + qi] = (m_used + __log2f(l)) * 0.69314718055994531f;
    }
  }

  tc_fence_before();
  __syncthreads();
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
