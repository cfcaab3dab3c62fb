// gemm.cuh -- bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// C[M,N] = A[M,K] . B[K,N] (+ fused epilogue), fp32 accumulation in TMEM.
// Either operand may be K-major or MN-major in HBM, so one kernel serves
// matmul_fwd (A K-major, B MN-major), dlhs = dout . rhs^T (B K-major) and
// drhs = lhs^T . dout (A and B MN-major) without any transpose pass.
//
// Persistent, warp-specialised CTA of 6 warps, one CTA per SM:
//   warp 0      TMA producer: STAGES-deep ring of (A 128x64, B BNx64) bf16 tiles,
//               128-byte swizzle, one mbarrier "full" and "empty" per stage.
//   warp 1      TMEM allocator + tcgen05.mma issuer (M=128, N=BN, K=16): the whole warp runs
//               the loop, one elected lane issues.
//   warps 2-5   epilogue: tcgen05.ld of the fp32 accumulator (one TMEM lane per
//               thread), fused RMSNorm row scale / bias / residual / SwiGLU, bf16 or f32
//               store, optionally the row sums of squares of what it stored.
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue
// of tile i overlaps the main loop of tile i+1.
#pragma once

#include "sm100.cuh"

namespace beacon {

// Every accumulator of row r is first multiplied by out_scale and, when the GEMM carries
// an RMSNorm (row_rms or row_sumsq set), by 1 / rms[r]; then the epilogue applies.
enum GemmEpilogue : int {
  kEpiStore = 0,       // out = acc
  kEpiBias = 1,        // out = acc + bias[col]
  kEpiResidual = 3,    // out = acc + residual[row, col]
  kEpiSwiglu = 4,      // out[:, j] = silu(acc_gate[:, j]) * acc_up[:, j]; B = [Wg | Wu] per tile
  kEpiSwigluSave = 5,  // kEpiSwiglu, and the gate and up values themselves to aux_g, aux_u
  // SwiGLU derivative of acc = dh = dy Wd^T, with g, u read from aux_g, aux_u:
  //   out[row, col]          = dgate = dh * u * s * (1 + g (1 - s)),  s = sigmoid(g)
  //   out[row, dup_off + col] = dup  = dh * g * s
  kEpiSwigluBwd = 6,
};
__host__ __device__ constexpr bool epi_tile_pairs(int epi) { return epi == kEpiSwiglu || epi == kEpiSwigluSave; }

struct GemmParams {
  int M, N, K;            // N: output columns (SwiGLU: F, the hidden width)
  int tiles_m, tiles_n;
  void* out;
  long long ldo;          // output row stride, elements
  int out_f32;            // 1: float32 output, 0: bf16 output
  int epi;
  int aux_f32;            // 1: bias / residual are float32, 0: bf16
  const void* bias;       // [N]
  const void* residual;   // [M, ldr]
  long long ldr;
  float out_scale;        // every accumulator is multiplied by it first (dequantisation scale; 1 = none)
  const float* out_scale_dev;  // when set, also by *out_scale_dev (a scale the device produced)
  // RMSNorm folded into the GEMM: rmsnorm(x) W = diag(1 / rms) . x . (diag(g) W), so the
  // GEMM reads raw x and the gain-folded weights and scales row r by 1 / rms[r], with
  //   rms[r] = row_rms[r]                                  when row_rms is set, else
  //   rms[r] = sqrt(row_sumsq[r] / row_dim + row_eps)      when row_sumsq is set.
  const float* row_rms;
  const float* row_sumsq;
  float row_dim, row_eps;
  // When set, the epilogue adds the sum of squares of the values it stores in row r
  // (after bf16 rounding) to out_sumsq[r]: the statistic of the next RMSNorm, accumulated
  // over the column tiles with one atomic add per row and tile.
  float* out_sumsq;
  // SwiGLU backward (bf16): kEpiSwigluSave writes gate / up here, kEpiSwigluBwd reads
  // them; [M, ld_aux].  kEpiSwigluBwd writes dup at column offset dup_off of out.
  void* aux_g;
  void* aux_u;
  long long ld_aux;
  long long dup_off;
  // Column split of the output: columns >= n_split go to out2 (column - n_split), same ldo.
  int n_split;
  void* out2;
  // K split of B: K-tiles at k >= k_split read the second B tensor map at k - k_split
  // (C = [A1 | A2] . [B1 ; B2] as one GEMM; k_split a multiple of 64).
  int k_split;
  // Head scatter (hd > 0): output column c of row r = b*seq + s is stored head-major,
  // [B, heads, seq, hd], into `out` for c < hq*hd, then `out_k`, then `out_v` (kv heads
  // each).  hd is a multiple of 32, so every 32-column chunk lands contiguously.
  int sc_seq, sc_hd, sc_hq, sc_hkv;
  void* out_k;
  void* out_v;
};

__device__ __forceinline__ float gemm_aux(const void* base, long long idx, int is_f32) {
  return is_f32 ? reinterpret_cast<const float*>(base)[idx]
                : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
}

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;  // one 128-byte swizzle row of bf16
  static constexpr int STAGES = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = BN * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * BN;  // power of two: 512 / 256 / 128
  static constexpr size_t SMEM_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
  static constexpr int THREADS = 192;
};

__device__ __forceinline__ float silu_f(float z) { return z / (1.0f + __expf(-z)); }

// The factor every accumulator of `row` is multiplied by before the epilogue.
__device__ __forceinline__ float gemm_row_factor(const GemmParams& p, int row) {
  float s = p.out_scale;
  if (p.out_scale_dev != nullptr) s *= *p.out_scale_dev;
  if (row < p.M) {
    if (p.row_rms != nullptr) s *= 1.0f / p.row_rms[row];
    else if (p.row_sumsq != nullptr) s *= 1.0f / sqrtf(p.row_sumsq[row] / p.row_dim + p.row_eps);
  }
  return s;
}

// Apply the epilogue to 32 consecutive columns [col0, col0+32) of one row (already
// scaled by gemm_row_factor) and store; returns the sum of squares of the stored values
// when p.out_sumsq is set (0 otherwise).
__device__ __forceinline__ float gemm_store_chunk(const GemmParams& p, int row, int col0, float (&v)[32]) {
  if (row >= p.M) return 0.0f;
  if (p.epi == kEpiBias && p.bias != nullptr) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < p.N) v[j] += gemm_aux(p.bias, col0 + j, p.aux_f32);
  }
  bool full = (col0 + 32 <= p.N);
  if (p.epi == kEpiResidual) {
    const long long rbase = (long long)row * p.ldr;
    if (!p.aux_f32 && full && (p.ldr & 7) == 0 && (col0 & 7) == 0 &&
        (reinterpret_cast<uintptr_t>(p.residual) & 15) == 0) {
      const uint4* r4 = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.residual) + rbase + col0);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 w = __ldg(r4 + j);
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          v[8 * j + 2 * e] += __uint_as_float(u[e] << 16);
          v[8 * j + 2 * e + 1] += __uint_as_float(u[e] & 0xffff0000u);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.N) v[j] += gemm_aux(p.residual, rbase + col0 + j, p.aux_f32);
    }
  }
  void* base = p.out;
  long long off = (long long)row * p.ldo + col0;
  long long ld = p.ldo;
  if (p.out2 != nullptr && col0 >= p.n_split) {  // chunks never straddle n_split (a multiple of 32)
    base = p.out2;
    off -= p.n_split;
  }
  if (p.sc_hd > 0) {
    int head = col0 / p.sc_hd, nh = p.sc_hq;
    if (head >= p.sc_hq) {
      head -= p.sc_hq;
      nh = p.sc_hkv;
      base = p.out_k;
      if (head >= p.sc_hkv) {
        head -= p.sc_hkv;
        base = p.out_v;
      }
    }
    const int bb = row / p.sc_seq, s = row - bb * p.sc_seq;
    off = (((long long)bb * nh + head) * p.sc_seq + s) * p.sc_hd + (col0 % p.sc_hd);
    ld = 0;  // chunks never straddle a head: the vector path's alignment holds
    full = true;
  }
  float ss = 0.0f;
  if (p.out_f32) {
    float* o = reinterpret_cast<float*>(base) + off;
    if (full && ((ld & 3) == 0)) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.N) o[j] = v[j];
    }
    if (p.out_sumsq != nullptr)
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.N) ss = fmaf(v[j], v[j], ss);
  } else {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(base) + off;
    if (p.out_sumsq != nullptr) {  // the statistic of what is stored: bf16-rounded values
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        v[j] = __bfloat162float(__float2bfloat16_rn(v[j]));
        if (col0 + j < p.N) ss = fmaf(v[j], v[j], ss);
      }
    }
    if (full && ((ld & 7) == 0)) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 w;
        w.x = pack_bf16x2(v[j + 0], v[j + 1]);
        w.y = pack_bf16x2(v[j + 2], v[j + 3]);
        w.z = pack_bf16x2(v[j + 4], v[j + 5]);
        w.w = pack_bf16x2(v[j + 6], v[j + 7]);
        *reinterpret_cast<uint4*>(o + j) = w;
      }
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.N) o[j] = __float2bfloat16_rn(v[j]);
    }
  }
  return ss;
}

// 32 bf16 values of row `row` at [col0, col0+32) of `base` (row stride ld), zero past n.
__device__ __forceinline__ void gemm_load_bf16_chunk(const void* base, long long ld, int row, int col0, int n,
                                                     float (&v)[32]) {
  const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(base) + (long long)row * ld + col0;
  if (col0 + 32 <= n) {  // rows 16-byte aligned (ld % 8 == 0, col0 % 32 == 0)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(src) + q);
      const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[8 * q + 2 * e] = __uint_as_float(u[e] << 16);
        v[8 * q + 2 * e + 1] = __uint_as_float(u[e] & 0xffff0000u);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (col0 + j < n) ? __bfloat162float(src[j]) : 0.0f;
  }
}

// 32 values to row `row`, columns [col0, col0+32) of a bf16 matrix (row stride ld), rounded;
// columns at or past n are not written.
__device__ __forceinline__ void gemm_store_bf16_chunk(void* base, long long ld, int row, int col0, int n,
                                                      const float (&v)[32]) {
  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(base) + (long long)row * ld + col0;
  if (col0 + 32 <= n) {
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      uint4 w;
      w.x = pack_bf16x2(v[j + 0], v[j + 1]);
      w.y = pack_bf16x2(v[j + 2], v[j + 3]);
      w.z = pack_bf16x2(v[j + 4], v[j + 5]);
      w.w = pack_bf16x2(v[j + 6], v[j + 7]);
      *reinterpret_cast<uint4*>(dst + j) = w;
    }
  } else {
    for (int j = 0; j < 32; ++j)
      if (col0 + j < n) dst[j] = __float2bfloat16_rn(v[j]);
  }
}

// kEpiSwigluBwd for 32 columns of dh = dy Wd^T (already scaled): the SwiGLU derivative
// with the recomputed gate / up, dgate to out and dup to out + dup_off (bf16).
__device__ __forceinline__ void gemm_store_swiglu_bwd(const GemmParams& p, int row, int col0, const float (&dh)[32]) {
  if (row >= p.M) return;
  float g[32], u[32];
  gemm_load_bf16_chunk(p.aux_g, p.ld_aux, row, col0, p.N, g);
  gemm_load_bf16_chunk(p.aux_u, p.ld_aux, row, col0, p.N, u);
  float dg[32], du[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float s = 1.0f / (1.0f + __expf(-g[j]));
    dg[j] = dh[j] * u[j] * s * (1.0f + g[j] * (1.0f - s));
    du[j] = dh[j] * g[j] * s;
  }
  gemm_store_bf16_chunk(p.out, p.ldo, row, col0, p.N, dg);
  gemm_store_bf16_chunk(reinterpret_cast<__nv_bfloat16*>(p.out) + p.dup_off, p.ldo, row, col0, p.N, du);
}

// The epilogue of one accumulator tile for one thread (one TMEM lane = output row `row`):
// BN fp32 columns at TMEM address `tbase`, column tile `tn`.  With tile pairs (SwiGLU) the
// first BN/2 columns are the gate and the last BN/2 the up projection of BN/2 outputs.
template <int BN>
__device__ __forceinline__ void gemm_epilogue_tile(const GemmParams& p, int row, uint32_t tbase, int tn, bool pairs) {
  const float rs = gemm_row_factor(p, row);
  float ss = 0.0f;
  if (!pairs) {
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(tbase + c * 32, r);
      tmem_wait_ld();
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * rs;
      const int col0 = tn * BN + c * 32;
      if (col0 < p.N) {
        if (p.epi == kEpiSwigluBwd)
          gemm_store_swiglu_bwd(p, row, col0, v);
        else
          ss += gemm_store_chunk(p, row, col0, v);
      }
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < BN / 64; ++c) {
      uint32_t g[32], u[32];
      tmem_ld32(tbase + c * 32, g);
      tmem_ld32(tbase + BN / 2 + c * 32, u);
      tmem_wait_ld();
      float gv[32], uv[32], v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        gv[j] = __uint_as_float(g[j]) * rs;
        uv[j] = __uint_as_float(u[j]) * rs;
        v[j] = silu_f(gv[j]) * uv[j];
      }
      const int col0 = tn * (BN / 2) + c * 32;
      if (col0 < p.N && row < p.M) {
        if (p.epi == kEpiSwigluSave) {
          gemm_store_bf16_chunk(p.aux_g, p.ld_aux, row, col0, p.N, gv);
          gemm_store_bf16_chunk(p.aux_u, p.ld_aux, row, col0, p.N, uv);
        }
        ss += gemm_store_chunk(p, row, col0, v);
      }
    }
  }
  if (p.out_sumsq != nullptr && row < p.M) atomicAdd(p.out_sumsq + row, ss);
}

// Fault-site codes (g_beacon_status[1]) for the GEMM's waits.
enum : unsigned int {
  kSiteGemmEmpty = 0x101,
  kSiteGemmTmemEmpty = 0x102,
  kSiteGemmFull = 0x103,
  kSiteGemmTmemFull = 0x104,
  kSiteGemmDrain = 0x105,
};

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(192, 1)
    k_gemm_bf16_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmB2, const GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int BM = Cfg::BM, BK = Cfg::BK, STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * Cfg::B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;  // [2]
  uint64_t* tempty = tfull + 2;      // [2]
  uint64_t* drain = tempty + 2;      // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);  // one arrive per epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (epi_tile_pairs(p.epi) || p.k_split > 0) tma_prefetch_desc(&tmB2);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.tiles_m * p.tiles_n;
  const int ktiles = (p.K + BK - 1) / BK;
  const bool swiglu = epi_tile_pairs(p.epi);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, issued_parity = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int tm = tile / p.tiles_n, tn = tile % p.tiles_n;
        for (int kt = 0; kt < ktiles; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteGemmEmpty)) {
            ok = false;
            break;
          }
          uint64_t* fb = &full[stage];
          mbar_arrive_expect_tx(fb, Cfg::STAGE_BYTES);
          uint8_t* a = sA + stage * Cfg::A_BYTES;
          uint8_t* b = sB + stage * Cfg::B_BYTES;
          const int k0 = kt * BK;
          if constexpr (!A_MN) {
            tma_load_2d(a, &tmA, fb, k0, tm * BM);
          } else {
            tma_load_2d(a, &tmA, fb, tm * BM, k0);
            tma_load_2d(a + 64 * BK * 2, &tmA, fb, tm * BM + 64, k0);
          }
          if (!swiglu) {
            // K split: the second half of K reads the second B tensor
            const bool second = p.k_split > 0 && k0 >= p.k_split;
            const CUtensorMap* mb = second ? &tmB2 : &tmB;
            const int kb = second ? k0 - p.k_split : k0;
            if constexpr (!B_MN) {
              tma_load_2d(b, mb, fb, kb, tn * BN);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j) tma_load_2d(b + j * 64 * BK * 2, mb, fb, tn * BN + j * 64, kb);
            }
          } else {
            const int n0 = tn * (BN / 2);
            if constexpr (!B_MN) {
              tma_load_2d(b, &tmB, fb, k0, n0);
              tma_load_2d(b + (BN / 2) * 128, &tmB2, fb, k0, n0);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 128; ++j) {
                tma_load_2d(b + j * 64 * BK * 2, &tmB, fb, n0 + j * 64, k0);
                tma_load_2d(b + (j + BN / 128) * 64 * BK * 2, &tmB2, fb, n0 + j * 64, k0);
              }
            }
          }
          issued |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let every TMA copy already in flight land before the CTA can exit.
        volatile int no_abort = 0;
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) mbar_wait(&full[s], (issued_parity >> s) & 1u, &no_abort, kSiteGemmDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop and waits; one elected lane issues. A lane-confined issuer
    // loses issue slots to the epilogue warp sharing its SM sub-partition.
    {
      const bool issuer = elect_one();
      constexpr uint32_t idesc = make_idesc_f16(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!warp_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, kSiteGemmTmemEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        for (int kt = 0; kt < ktiles; ++kt) {
          if (!warp_wait(&full[stage], phase, abort_flag, kSiteGemmFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? make_sdesc_sw128(a_addr + kk * 2048, 64 * BK * 2, 1024)
                                     : make_sdesc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? make_sdesc_sw128(b_addr + kk * 2048, 64 * BK * 2, 1024)
                                     : make_sdesc_sw128(b_addr + kk * 32, 16, 1024);
            if (issuer) umma_f16_ss(d, ad, bd, idesc, (kt | kk) != 0 ? 1u : 0u);
          }
          if (issuer) umma_commit(&empty[stage]);  // frees the smem stage once these MMAs have read it
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (issuer) umma_commit(&tfull[acc]);  // accumulator ready for the epilogue
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      // Drain: every MMA this thread issued has finished before TMEM is freed.
      if (issuer) umma_commit(drain);
      volatile int no_abort = 0;
      warp_wait(drain, 0, &no_abort, kSiteGemmDrain);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const uint32_t q = warp & 3u;  // TMEM lane quarter this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int tm = tile / p.tiles_n, tn = tile % p.tiles_n;
      const bool got = mbar_wait(&tfull[acc], acc_phase, abort_flag, kSiteGemmTmemFull);
      if (!__all_sync(0xffffffffu, got)) break;  // warp-uniform: tcgen05.ld below is warp-collective
      tc_fence_after();
      const int row = tm * BM + (int)(q * 32 + lane);
      gemm_epilogue_tile<BN>(p, row, tmem_base + ((q * 32u) << 16) + (uint32_t)(acc * BN), tn, swiglu);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// 2-SM variant: a cluster of two CTAs computes a 256xBN tile with
// tcgen05.mma.cta_group::2 (M = 256 over the pair).  Each CTA TMA-loads its own 128 rows
// of A and its own BN/2-column half of B (for SwiGLU, BN = 256: CTA 0 the gate columns,
// CTA 1 the up columns), so every SM streams half the B operand a 1-SM 128xBN tile would,
// and the pair's loads complete on the leader CTA's barrier.  Only the leader issues MMAs;
// each CTA's TMEM receives its 128 accumulator rows and its own epilogue warps drain
// them.  No load uses multicast.  BN = 256 is the general tile; BN = 128 (256x128 pair
// tiles) serves narrow outputs such as a column shard of N = 512, where 256x256 tiles
// would leave half the SMs idle and 1-SM 128x128 tiles need more operand bytes per clock
// than TMA delivers to an SM.
// ---------------------------------------------------------------------------
template <int BN_>
struct GemmCfg2 {
  static constexpr int BM = 128, BN = BN_, BK = 64, STAGES = BN_ == 256 ? 6 : 8;
  static constexpr uint32_t A_BYTES = BM * BK * 2;           // this CTA's 128 rows of A
  static constexpr uint32_t B_BYTES = (BN / 2) * BK * 2;     // this CTA's half of B
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr size_t SMEM_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
  static constexpr int THREADS = 192;
};

template <bool A_MN, bool B_MN, int BN = 256>
__global__ void __launch_bounds__(192, 1)
    k_gemm_bf16_tc2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmB2, const GemmParams p) {
  using Cfg = GemmCfg2<BN>;
  static_assert(BN == 256 || BN == 128, "pair tiles of 256 x 256 or 256 x 128");
  constexpr int BK = Cfg::BK, STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * Cfg::B_BYTES);  // used in the leader
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;  // [2]
  uint64_t* tempty = tfull + 2;      // [2] used in the leader: 4 epilogue warps x 2 CTAs
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = (int)(blockIdx.x >> 1), n_clusters = (int)(gridDim.x >> 1);
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
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
    tma_prefetch_desc(&tmB);
    if (epi_tile_pairs(p.epi) || p.k_split > 0) tma_prefetch_desc(&tmB2);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrive or commit
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.tiles_m * p.tiles_n;  // tiles of 256 x BN (SwiGLU: 256 x 128 outputs)
  const int ktiles = (p.K + BK - 1) / BK;
  const bool swiglu = BN == 256 && epi_tile_pairs(p.epi);

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
        const CUtensorMap* mb_tile = (swiglu && rank == 1) ? &tmB2 : &tmB;
        const int n0 = swiglu ? tn * 128 : tn * BN + (BN / 2) * (int)rank;
        for (int kt = 0; kt < ktiles; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteGemmEmpty)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
          const uint32_t lb = cluster_map(&full[stage], 0);  // the leader's barrier
          uint8_t* a = sA + stage * Cfg::A_BYTES;
          uint8_t* b = sB + stage * Cfg::B_BYTES;
          const int k0 = kt * BK;
          if constexpr (!A_MN) {
            tma_load_2d_pair(a, &tmA, lb, k0, m0);
          } else {
            tma_load_2d_pair(a, &tmA, lb, m0, k0);
            tma_load_2d_pair(a + 64 * BK * 2, &tmA, lb, m0 + 64, k0);
          }
          // K split: the second half of K reads the second B tensor
          const bool second = !swiglu && p.k_split > 0 && k0 >= p.k_split;
          const CUtensorMap* mb = second ? &tmB2 : mb_tile;
          const int kb = second ? k0 - p.k_split : k0;
          if constexpr (!B_MN) {
            tma_load_2d_pair(b, mb, lb, kb, n0);  // BN/2 rows of B^T (the tensor map's box)
          } else {
#pragma unroll
            for (int h = 0; h < BN / 128; ++h) tma_load_2d_pair(b + h * 64 * BK * 2, mb, lb, n0 + 64 * h, kb);
          }
          issued |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && leader) {
        // the leader's barriers count both CTAs' copies: let every one in flight land
        volatile int no_abort = 0;
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) mbar_wait(&full[s], (issued_parity >> s) & 1u, &no_abort, kSiteGemmDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA only)
    // The whole warp runs the loop and waits; one elected lane issues.
    if (leader) {
      const bool issuer = elect_one();
      constexpr uint32_t idesc = make_idesc_f16(256, Cfg::BN, A_MN, B_MN);
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
          if (!warp_wait(&full[stage], phase, abort_flag, kSiteGemmFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? make_sdesc_sw128(a_addr + kk * 2048, 64 * BK * 2, 1024)
                                     : make_sdesc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? make_sdesc_sw128(b_addr + kk * 2048, 64 * BK * 2, 1024)
                                     : make_sdesc_sw128(b_addr + kk * 32, 16, 1024);
            if (issuer) umma_f16_ss_pair(d, ad, bd, idesc, (kt | kk) != 0 ? 1u : 0u);
          }
          if (issuer) umma_commit_pair(&empty[stage]);  // both CTAs' stages are free once these MMAs read them
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
  } else {
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
      gemm_epilogue_tile<Cfg::BN>(p, row, tmem_base + ((q * 32u) << 16) + (uint32_t)(acc * Cfg::BN), tn, swiglu);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
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

// ---------------------------------------------------------------------------
// Exact-FP32 SIMT GEMM (FFMA only, no TF32) for f32 operands and for bf16 shapes
// the TMA path cannot describe (row strides not a multiple of 16 bytes).
// A(m,k) = A[m*sam + k*sak], B(k,n) = B[k*sbk + n*sbn]; 64x64 tile, 4x4 per thread.
// ---------------------------------------------------------------------------
template <typename TIn>
__device__ __forceinline__ float to_f(TIn x);
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename TIn>
__global__ void __launch_bounds__(256)
    k_gemm_simt(const TIn* __restrict__ A, long long sam, long long sak, const TIn* __restrict__ B, long long sbk,
                long long sbn, const GemmParams p) {
  __shared__ float As[16][64 + 1];
  __shared__ float Bs[16][64 + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < p.K; k0 += 16) {
    for (int e = threadIdx.x; e < 16 * 64; e += 256) {
      const int kk = e / 64, mm = e % 64;
      const int m = m0 + mm, k = k0 + kk;
      As[kk][mm] = (m < p.M && k < p.K) ? to_f(A[m * sam + k * sak]) : 0.0f;
      const int n = n0 + mm;
      Bs[kk][mm] = (n < p.N && k < p.K) ? to_f(B[k * sbk + n * sbn]) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= p.M) continue;
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= p.N) continue;
      float v = acc[i][j] * gemm_row_factor(p, m);
      if (p.epi == kEpiBias && p.bias) v += gemm_aux(p.bias, n, p.aux_f32);
      if (p.epi == kEpiResidual) v += gemm_aux(p.residual, m * p.ldr + n, p.aux_f32);
      if (p.out_f32)
        reinterpret_cast<float*>(p.out)[m * p.ldo + n] = v;
      else
        reinterpret_cast<__nv_bfloat16*>(p.out)[m * p.ldo + n] = __float2bfloat16_rn(v);
    }
  }
}

}  // namespace beacon
