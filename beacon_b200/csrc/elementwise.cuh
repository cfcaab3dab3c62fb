// elementwise.cuh -- residual add, casts, RMSNorm and LayerNorm forward/backward.
//
// All HBM-bound: 128-bit vectorised, coalesced loads and stores, fp32 math,
// warp-shuffle reductions.  The dtype codecs restate the reference's bit-level
// rules (crates/beacon-core/src/dtype.rs) so casts are bit-exact with it.
#pragma once

#include "sm100.cuh"

namespace beacon {

// ---------------------------------------------------------------------------
// dtype codecs (device), dtype.rs:58-66 (bf16) and dtype.rs:138-209 (fp8 e4m3)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint16_t bf16_bits_from_f32(float x) {
  const uint32_t bits = __float_as_uint(x);
  if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x0040u);
  const uint32_t bias = 0x7fffu + ((bits >> 16) & 1u);
  return (uint16_t)((bits + bias) >> 16);
}

// Rust f32::round is half-away-from-zero; ties are detected inside an
// f32::EPSILON window and sent to the even neighbour (dtype.rs:197-209).
__device__ __forceinline__ float round_half_even_window(float x) {
  const float r = roundf(x);
  if (fabsf(x - floorf(x) - 0.5f) < 1.1920929e-7f) {
    const float down = floorf(x);
    return ((((long long)down) % 2) == 0) ? down : down + 1.0f;
  }
  return r;
}

__device__ __forceinline__ uint8_t fp8e4m3_from_f32(float x) {
  if (isnan(x)) return 0xff;
  const uint8_t sign_bit = signbit(x) ? 0x80 : 0x00;
  const float ax = fabsf(x);
  if (ax == 0.0f) return sign_bit;
  if (ax >= 448.0f) return (uint8_t)(sign_bit | 0x7e);
  if (ax < 0.015625f) {  // below 2^-6, the smallest normal: multiples of 2^-9
    float m = round_half_even_window(ax * 512.0f);
    if (m > 7.0f) m = 7.0f;
    return (uint8_t)(sign_bit | (uint8_t)m);
  }
  // floor(log2(ax)) of a normal float is its unbiased exponent; where a rounded
  // log2 would land on the next integer the mantissa rounds up to 8 below and
  // the exponent is bumped, giving the same code.
  int exp = (int)((__float_as_uint(ax) >> 23) & 0xff) - 127;
  if (exp < -6) exp = -6;
  const float frac = ax * __uint_as_float((uint32_t)(127 - exp) << 23) - 1.0f;  // ax / 2^exp, exact
  int mant = (int)round_half_even_window(frac * 8.0f);
  int biased = exp + 7;
  if (mant == 8) {
    mant = 0;
    biased += 1;
  }
  if (biased >= 0x0f && mant >= 0x07) return (uint8_t)(sign_bit | 0x7e);
  return (uint8_t)(sign_bit | (uint8_t)(biased << 3) | (uint8_t)mant);
}

__device__ __forceinline__ float fp8e4m3_to_f32(uint8_t b) {
  const float sign = (b & 0x80) ? -1.0f : 1.0f;
  const int exp = (b >> 3) & 0x0f;
  const int mant = b & 0x07;
  if (exp == 0x0f && mant == 0x07) return __uint_as_float(0x7fc00000u);
  if (exp == 0) return sign * (float)mant * 0.001953125f;  // 2^-9
  return sign * (1.0f + (float)mant * 0.125f) * __uint_as_float((uint32_t)(exp - 7 + 127) << 23);
}

// ---------------------------------------------------------------------------
// residual add / backward / casts: grid-stride, 16-byte vectors + scalar tail
// ---------------------------------------------------------------------------
__global__ void k_add_bf16(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ a,
                           const __nv_bfloat16* __restrict__ b, long long n) {
  const long long nvec = n / 8;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const uint4 va = reinterpret_cast<const uint4*>(a)[i];
    const uint4 vb = reinterpret_cast<const uint4*>(b)[i];
    const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&va);
    const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&vb);
    uint4 vo;
    __nv_bfloat162* po = reinterpret_cast<__nv_bfloat162*>(&vo);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 fa = __bfloat1622float2(pa[j]), fb = __bfloat1622float2(pb[j]);
      po[j] = __floats2bfloat162_rn(fa.x + fb.x, fa.y + fb.y);
    }
    reinterpret_cast<uint4*>(out)[i] = vo;
  }
  for (long long i = nvec * 8 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = __float2bfloat16_rn(__bfloat162float(a[i]) + __bfloat162float(b[i]));
}

__global__ void k_add_f32(float* __restrict__ out, const float* __restrict__ a, const float* __restrict__ b,
                          long long n) {
  const long long nvec = n / 4;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const float4 va = reinterpret_cast<const float4*>(a)[i];
    const float4 vb = reinterpret_cast<const float4*>(b)[i];
    reinterpret_cast<float4*>(out)[i] = make_float4(va.x + vb.x, va.y + vb.y, va.z + vb.z, va.w + vb.w);
  }
  for (long long i = nvec * 4 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = a[i] + b[i];
}

// d_a = d_b = d_out, for any element size: copy 16-byte vectors then bytes.
__global__ void k_fanout2(uint8_t* __restrict__ da, uint8_t* __restrict__ db, const uint8_t* __restrict__ src,
                          long long nbytes) {
  const long long nvec = nbytes / 16;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const uint4 v = reinterpret_cast<const uint4*>(src)[i];
    if (da) reinterpret_cast<uint4*>(da)[i] = v;
    if (db) reinterpret_cast<uint4*>(db)[i] = v;
  }
  for (long long i = nvec * 16 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nbytes; i += stride) {
    if (da) da[i] = src[i];
    if (db) db[i] = src[i];
  }
}

// kind: 0 f32->fp8, 1 fp8->f32, 2 f32->bf16, 3 bf16->f32 (CastKind order)
__global__ void k_cast(void* __restrict__ dst, const void* __restrict__ src, long long n, int kind) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    switch (kind) {
      case 0:
        reinterpret_cast<uint8_t*>(dst)[i] = fp8e4m3_from_f32(reinterpret_cast<const float*>(src)[i]);
        break;
      case 1:
        reinterpret_cast<float*>(dst)[i] = fp8e4m3_to_f32(reinterpret_cast<const uint8_t*>(src)[i]);
        break;
      case 2:
        reinterpret_cast<uint16_t*>(dst)[i] = bf16_bits_from_f32(reinterpret_cast<const float*>(src)[i]);
        break;
      default:
        reinterpret_cast<float*>(dst)[i] =
            __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(src)[i] << 16);
        break;
    }
  }
}

// ---------------------------------------------------------------------------
// Embedding lookup (crates/beacon-cuda/src/elementwise.rs:67-95): out[t, :] = table[idx[t], :]
// with u32 indices; the backward adds d_out[t, :] into d_table[idx[t], :] (d_table is
// ReadWrite in the reference's own test, elementwise.rs:185).  An index at or beyond
// `vocab` is not followed: its output row is written as zeros (forward) or skipped
// (backward), and the fault word records kFaultIndex once per launch site.
// ---------------------------------------------------------------------------
constexpr unsigned int kFaultIndex = 3;

__device__ __forceinline__ float elem_ld(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ float elem_ld(const float* p) { return *p; }
__device__ __forceinline__ void elem_st(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
__device__ __forceinline__ void elem_st(float* p, float v) { *p = v; }

// One warp per token row; 16-byte vectors when `vec` (rows 16-byte aligned, dim * es % 16 == 0).
template <typename T>
__global__ void __launch_bounds__(256) k_embedding_fwd(T* __restrict__ out, const T* __restrict__ table,
                                                       const uint32_t* __restrict__ idx, long long tokens, int dim,
                                                       long long vocab, int vec, unsigned int site) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long t = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < tokens; t += warps) {
    const uint32_t r = idx[t];
    T* o = out + t * dim;
    if ((long long)r >= vocab) {
      if (lane == 0) record_fault(kFaultIndex, site);
      for (int e = lane; e < dim; e += 32) o[e] = T(0.0f);
      continue;
    }
    const T* src = table + (long long)r * dim;
    if (vec) {
      const int nv = dim * (int)sizeof(T) / 16;
      for (int v = lane; v < nv; v += 32) reinterpret_cast<uint4*>(o)[v] = reinterpret_cast<const uint4*>(src)[v];
    } else {
      for (int e = lane; e < dim; e += 32) o[e] = src[e];
    }
  }
}

__device__ __forceinline__ void atomic_add_elem(float* p, float v) { atomicAdd(p, v); }
__device__ __forceinline__ void atomic_add_elem(__nv_bfloat16* p, float v) { atomicAdd(p, __float2bfloat16_rn(v)); }

// One warp per token row: d_table[idx[t], e] += d_out[t, e] (atomic adds: tokens sharing an
// index add in any order).
template <typename T>
__global__ void __launch_bounds__(256) k_embedding_bwd(T* __restrict__ d_table, const T* __restrict__ d_out,
                                                       const uint32_t* __restrict__ idx, long long tokens, int dim,
                                                       long long vocab, unsigned int site) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long t = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < tokens; t += warps) {
    const uint32_t r = idx[t];
    if ((long long)r >= vocab) {
      if (lane == 0) record_fault(kFaultIndex, site);
      continue;
    }
    T* dst = d_table + (long long)r * dim;
    const T* src = d_out + t * dim;
    for (int e = lane; e < dim; e += 32) atomic_add_elem(dst + e, elem_ld(src + e));
  }
}

// ---------------------------------------------------------------------------
// Dropout (crates/beacon-cuda/src/elementwise.rs:97-118).  Element i is kept when
// u_i >= p, u_i = (splitmix64(seed, i) >> 40) / 2^24 (the counter-based generator the
// synthetic inputs use, so the mask depends on (seed, i) only, not on the launch shape).
// mask[i] holds the multiplier, 1 / (1 - p) for a kept element and 0 for a dropped one,
// rounded to the data type; out = input * mask and the backward, which the reference
// calls without p (elementwise.rs:110-118), is d_in = d_out * mask.  p >= 1 drops all.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t splitmix64_at(uint64_t seed, uint64_t i) {
  uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ULL;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

template <typename T>
__global__ void k_dropout_fwd(T* __restrict__ out, T* __restrict__ mask, const T* __restrict__ in, long long n,
                              float p, unsigned long long seed) {
  const float keep_scale = p < 1.0f ? 1.0f / (1.0f - p) : 0.0f;
  const T m_keep = T(keep_scale);
  const float mk = elem_ld(&m_keep);
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float u = (float)(splitmix64_at(seed, (uint64_t)i) >> 40) * (1.0f / 16777216.0f);
    const bool keep = p < 1.0f && u >= p;
    mask[i] = keep ? m_keep : T(0.0f);
    elem_st(out + i, keep ? elem_ld(in + i) * mk : 0.0f);
  }
}

template <typename T>
__global__ void k_dropout_bwd(T* __restrict__ d_in, const T* __restrict__ d_out, const T* __restrict__ mask,
                              long long n) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    elem_st(d_in + i, elem_ld(d_out + i) * elem_ld(mask + i));
}

// ---------------------------------------------------------------------------
// fp32 master -> fp8 e4m3 weights with one scale per tensor
//   amax = max |x| (NaN ignored), scale = amax / 448 (1 when amax is 0),
//   q = F8E4M3::from_f32(x * (448 / amax)), so that x ~ decode(q) * scale.
// k_absmax folds each CTA's maximum into *amax_bits (the float's bits: for values >= 0
// the unsigned order is the float order; the word starts at 0); k_quantize_fp8 reads it.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_absmax(unsigned int* __restrict__ amax_bits, const float* __restrict__ x,
                                                long long n) {
  __shared__ float red[8];
  float m = 0.0f;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long nvec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) ? n / 4 : 0;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  for (long long i = nvec * 4 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    m = fmaxf(m, fabsf(x[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = red[0];
    for (int w = 1; w < 8; ++w) b = fmaxf(b, red[w]);
    atomicMax(amax_bits, __float_as_uint(b));
  }
}

__global__ void __launch_bounds__(256) k_quantize_fp8(uint8_t* __restrict__ q, float* __restrict__ scale,
                                                      const float* __restrict__ amax, const float* __restrict__ x,
                                                      long long n) {
  const float a = *amax;
  const float inv = a > 0.0f ? 448.0f / a : 1.0f;
  if (blockIdx.x == 0 && threadIdx.x == 0) *scale = a > 0.0f ? a / 448.0f : 1.0f;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    q[i] = fp8e4m3_from_f32(x[i] * inv);
}

// fp8 e4m3 -> bf16, 16 elements per thread-step (every e4m3 value is exact in bf16).
__global__ void k_fp8_to_bf16(uint16_t* __restrict__ dst, const uint8_t* __restrict__ src, long long n) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long nvec = n / 16;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const uint4 in = reinterpret_cast<const uint4*>(src)[i];
    const uint8_t* b = reinterpret_cast<const uint8_t*>(&in);
    uint4 o[2];
    uint16_t* h = reinterpret_cast<uint16_t*>(o);
#pragma unroll
    for (int j = 0; j < 16; ++j) h[j] = (uint16_t)(__float_as_uint(fp8e4m3_to_f32(b[j])) >> 16);
    reinterpret_cast<uint4*>(dst)[2 * i] = o[0];
    reinterpret_cast<uint4*>(dst)[2 * i + 1] = o[1];
  }
  for (long long i = nvec * 16 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = (uint16_t)(__float_as_uint(fp8e4m3_to_f32(src[i])) >> 16);
}

// ---------------------------------------------------------------------------
// RMSNorm
// ---------------------------------------------------------------------------
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ float ldf(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ float ldf(const float* p) { return *p; }
__device__ __forceinline__ void stf(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
__device__ __forceinline__ void stf(float* p, float v) { *p = v; }

// Dropout (the draw and arithmetic of k_dropout_fwd / k_dropout_bwd above).
// The same draw and arithmetic, eight elements per thread with 16-byte loads and stores (the
// scalar kernel's 2-byte accesses and one hash per thread kept it at half of HBM speed);
// pointers 16-byte aligned.  The n % 8 tail is done by the first threads of CTA 0.
template <typename T>
__global__ void __launch_bounds__(256) k_dropout_fwd_vec(T* __restrict__ out, T* __restrict__ mask,
                                                         const T* __restrict__ in, long long n, float p,
                                                         unsigned long long seed) {
  const float keep_scale = p < 1.0f ? 1.0f / (1.0f - p) : 0.0f;
  const T m_keep = T(keep_scale);
  const float mk = elem_ld(&m_keep);
  const long long n8 = n / 8, stride = (long long)gridDim.x * blockDim.x;
  for (long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x; g < n8; g += stride) {
    const long long i0 = g * 8;
    float x[8], o[8], m[8];
    load8(in + i0, x);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float u = (float)(splitmix64_at(seed, (uint64_t)(i0 + j)) >> 40) * (1.0f / 16777216.0f);
      const bool keep = p < 1.0f && u >= p;
      m[j] = keep ? mk : 0.0f;
      o[j] = keep ? x[j] * mk : 0.0f;
    }
    store8(mask + i0, m);
    store8(out + i0, o);
  }
  if (blockIdx.x == 0 && threadIdx.x < n - n8 * 8) {
    const long long i = n8 * 8 + threadIdx.x;
    const float u = (float)(splitmix64_at(seed, (uint64_t)i) >> 40) * (1.0f / 16777216.0f);
    const bool keep = p < 1.0f && u >= p;
    mask[i] = keep ? m_keep : T(0.0f);
    elem_st(out + i, keep ? elem_ld(in + i) * mk : 0.0f);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) k_dropout_bwd_vec(T* __restrict__ d_in, const T* __restrict__ d_out,
                                                         const T* __restrict__ mask, long long n) {
  const long long n8 = n / 8, stride = (long long)gridDim.x * blockDim.x;
  for (long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x; g < n8; g += stride) {
    float a[8], b[8], o[8];
    load8(d_out + g * 8, a);
    load8(mask + g * 8, b);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = a[j] * b[j];
    store8(d_in + g * 8, o);
  }
  if (blockIdx.x == 0 && threadIdx.x < n - n8 * 8) {
    const long long i = n8 * 8 + threadIdx.x;
    elem_st(d_in + i, elem_ld(d_out + i) * elem_ld(mask + i));
  }
}


__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum for blockDim.x == 256; `red` holds 8 floats of shared memory.
__device__ __forceinline__ float block_sum_256(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (l < 8) ? red[l] : 0.0f;
  t = warp_sum(t);
  return t;
}

// WPR warps per bf16 row (norm.rs:20-31), each lane holding 8 x NCH values of the row from
// 16-byte loads (512 bytes per warp instruction; a row is WPR x NCH x 256 elements), grid-
// stride over rows in steps of the grid's row slots.  The sum of squares is a shuffle
// reduction (plus, for two warps per row, one exchange through shared memory behind a
// 64-thread named barrier), so no CTA-wide barrier holds the other rows back: every
// resident warp can have its row's loads in flight, where a CTA per row keeps about eight
// rows in flight per SM and none while it reduces.  x is read with the streaming
// (evict-first) hint and y stored with it; the weight row stays cached.  Two warps per
// 4096-wide row keep a lane at 8 chunks (one warp would need 16 and spill).
template <int NCH, int WPR>
__global__ void __launch_bounds__(256, 2) k_rmsnorm_fwd_warp(__nv_bfloat16* __restrict__ y, float* __restrict__ rms,
                                                             const __nv_bfloat16* __restrict__ x,
                                                             const __nv_bfloat16* __restrict__ w, long long rows,
                                                             int dim, float eps) {
  static_assert(WPR == 1 || WPR == 2, "one or two warps per row");
  __shared__ float part[8];
  const int lane = (int)(threadIdx.x & 31u), warp = (int)(threadIdx.x >> 5);
  const int slot = warp / WPR, sub = warp % WPR;  // row slot of the CTA, this warp's share of the row
  constexpr int SLOTS = 8 / WPR;
  const long long ns = (long long)gridDim.x * SLOTS;
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  for (long long r = (long long)blockIdx.x * SLOTS + slot; r < rows; r += ns) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + r * dim);
    uint4 u[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) u[c] = __ldcs(xr + (c * WPR + sub) * 32 + lane);
    float ss = 0.0f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[c]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
    ss = warp_sum(ss);
    if constexpr (WPR == 2) {
      if (lane == 0) part[warp] = ss;
      named_bar_sync(1 + slot, 64);
      ss = part[2 * slot] + part[2 * slot + 1];
      named_bar_sync(1 + slot, 64);  // both have read the pair's partials before the next row's
    }
    const float rr = sqrtf(ss / (float)dim + eps);
    const float inv = 1.0f / rr;
    if (lane == 0 && sub == 0) rms[r] = rr;
    uint4* yr = reinterpret_cast<uint4*>(y + r * dim);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int v = (c * WPR + sub) * 32 + lane;
      const uint4 gu = __ldg(wv + v);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[c]);
      const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&gu);
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]), g = __bfloat1622float2(gh[j]);
        o[j] = pack_bf16x2(f.x * inv * g.x, f.y * inv * g.y);
      }
      __stcs(yr + v, make_uint4(o[0], o[1], o[2], o[3]));
    }
  }
}

// One CTA of 256 threads per row (norm.rs:5-9 `rowwise`), grid-stride over rows.
// VEC: 8-element vectors per thread held in registers (dim <= 256*8*VEC).
template <typename T, int VEC>
__global__ void __launch_bounds__(256) k_rmsnorm_fwd(T* __restrict__ y, float* __restrict__ rms,
                                                     const T* __restrict__ x, const T* __restrict__ w,
                                                     long long rows, int dim, float eps) {
  __shared__ float red[8];
  const int nvec = dim / 8;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* xr = x + r * dim;
    float v[VEC][8];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi < nvec) {
        load8(xr + vi * 8, v[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = fmaf(v[i][j], v[i][j], ss);
      }
    }
    for (int e = nvec * 8 + threadIdx.x; e < dim; e += 256) {  // dim % 8 tail
      const float t = ldf(xr + e);
      ss = fmaf(t, t, ss);
    }
    ss = block_sum_256(ss, red);
    const float rr = sqrtf(ss / (float)dim + eps);
    const float inv = 1.0f / rr;
    if (threadIdx.x == 0) rms[r] = rr;
    T* yr = y + r * dim;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi < nvec) {
        float g[8], o[8];
        load8(w + vi * 8, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = v[i][j] * inv * g[j];
        store8(yr + vi * 8, o);
      }
    }
    for (int e = nvec * 8 + threadIdx.x; e < dim; e += 256) stf(yr + e, ldf(xr + e) * inv * ldf(w + e));
  }
}

// Row statistics of an RMSNorm whose scaling is folded into the GEMM that consumes the
// rows (rmsnorm(x) W = diag(1/rms) x (diag(g) W)): reads x once and writes only
// rms[r] = sqrt(mean(x[r]^2) + eps) (when rms != null) and the sum of squares (when
// sumsq != null), 4 or 8 bytes per row instead of a normalised copy of x.  One warp per
// row, vectors of 8 elements (16 bytes of bf16) four deep; `vec` rows are 16-byte aligned
// with dim % 8 == 0.
template <typename T>
__global__ void __launch_bounds__(256) k_rms_stats(float* __restrict__ rms, float* __restrict__ sumsq,
                                                   const T* __restrict__ x, long long rows, int dim, float eps,
                                                   int vec) {
  constexpr int EPV = 8;
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const T* xr = x + r * dim;
    float ss = 0.0f;
    if (vec) {
      const int nv = dim / EPV;
      int vi = lane;
      for (; vi + 96 < nv; vi += 128) {
        float a[4][8];
#pragma unroll
        for (int u = 0; u < 4; ++u) load8(xr + (vi + 32 * u) * EPV, a[u]);
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int j = 0; j < EPV; ++j) ss = fmaf(a[u][j], a[u][j], ss);
      }
      for (; vi < nv; vi += 32) {
        float a[8];
        load8(xr + vi * EPV, a);
#pragma unroll
        for (int j = 0; j < EPV; ++j) ss = fmaf(a[j], a[j], ss);
      }
    } else {
      for (int e = lane; e < dim; e += 32) {
        const float t = ldf(xr + e);
        ss = fmaf(t, t, ss);
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) {
      if (rms) rms[r] = sqrtf(ss / (float)dim + eps);
      if (sumsq) sumsq[r] = ss;
    }
  }
}

// w_out[i, j] = gain[i] * w[i, j], rounded to T: the RMSNorm gain folded into the rows
// (the input dimension) of the weight that follows the norm.  Once per weight version.
template <typename T>
__global__ void k_fold_gain(T* __restrict__ w_out, const T* __restrict__ gain, const T* __restrict__ w, long long k,
                            long long n) {
  const long long total = k * n;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x)
    stf(w_out + i, ldf(gain + i / n) * ldf(w + i));
}

// Generic fallback for any dim (two passes over the row, second from L1/L2).
template <typename T>
__global__ void __launch_bounds__(256) k_rmsnorm_fwd_any(T* __restrict__ y, float* __restrict__ rms,
                                                         const T* __restrict__ x, const T* __restrict__ w,
                                                         long long rows, int dim, float eps) {
  __shared__ float red[8];
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* xr = x + r * dim;
    float ss = 0.0f;
    for (int e = threadIdx.x; e < dim; e += 256) {
      const float t = ldf(xr + e);
      ss = fmaf(t, t, ss);
    }
    ss = block_sum_256(ss, red);
    const float rr = sqrtf(ss / (float)dim + eps);
    const float inv = 1.0f / rr;
    if (threadIdx.x == 0) rms[r] = rr;
    for (int e = threadIdx.x; e < dim; e += 256) stf(y + r * dim + e, ldf(xr + e) * inv * ldf(w + e));
  }
}

// Backward: dx per row; dweight partial sums per CTA into part[blockIdx.x, dim] (fp32).
template <typename T>
__global__ void __launch_bounds__(256) k_rmsnorm_bwd(T* __restrict__ dx, float* __restrict__ part,
                                                     const T* __restrict__ dy, const T* __restrict__ x,
                                                     const float* __restrict__ rms, const T* __restrict__ w,
                                                     long long rows, int dim) {
  __shared__ float red[8];
  const bool vec = (dim % 8) == 0;
  float* pr = part ? part + (long long)blockIdx.x * dim : nullptr;
  // zero this CTA's partial row
  if (pr)
    for (int e = threadIdx.x; e < dim; e += 256) pr[e] = 0.0f;
  __syncthreads();
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* xr = x + r * dim;
    const T* dyr = dy + r * dim;
    const float rr = rms[r];
    const float inv = 1.0f / rr;
    float dot = 0.0f;
    if (vec) {
      for (int vi = threadIdx.x; vi < dim / 8; vi += 256) {
        float a[8], b[8], g[8];
        load8(xr + vi * 8, a);
        load8(dyr + vi * 8, b);
        load8(w + vi * 8, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) dot = fmaf(g[j] * b[j], a[j], dot);
      }
    } else {
      for (int e = threadIdx.x; e < dim; e += 256) dot = fmaf(ldf(w + e) * ldf(dyr + e), ldf(xr + e), dot);
    }
    dot = block_sum_256(dot, red);
    const float c = dot * inv * inv * inv / (float)dim;
    T* dxr = dx + r * dim;
    if (vec) {
      for (int vi = threadIdx.x; vi < dim / 8; vi += 256) {
        float a[8], b[8], g[8], o[8];
        load8(xr + vi * 8, a);
        load8(dyr + vi * 8, b);
        load8(w + vi * 8, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = g[j] * b[j] * inv - a[j] * c;
        store8(dxr + vi * 8, o);
        if (pr) {
#pragma unroll
          for (int j = 0; j < 8; ++j) pr[vi * 8 + j] += b[j] * a[j] * inv;
        }
      }
    } else {
      for (int e = threadIdx.x; e < dim; e += 256) {
        const float a = ldf(xr + e), b = ldf(dyr + e);
        stf(dxr + e, ldf(w + e) * b * inv - a * c);
        if (pr) pr[e] += b * a * inv;
      }
    }
  }
}

// dweight[d] = sum over CTAs of part[cta, d]
template <typename T>
__global__ void k_colsum(T* __restrict__ out, const float* __restrict__ part, int nparts, int dim) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= dim) return;
  float s = 0.0f;
  for (int i = 0; i < nparts; ++i) s += part[(long long)i * dim + d];
  stf(out + d, s);
}

// dbias[n] = sum_rows dout[m, n]: CTA-partial column sums (fp32) then k_colsum.
template <typename T>
__global__ void __launch_bounds__(256) k_colsum_partial(float* __restrict__ part, const T* __restrict__ src,
                                                        long long rows, int cols) {
  for (int c = threadIdx.x; c < cols; c += 256) {
    float s = 0.0f;
    for (long long r = blockIdx.x; r < rows; r += gridDim.x) s += ldf(src + r * cols + c);
    part[(long long)blockIdx.x * cols + c] = s;
  }
}

// ---------------------------------------------------------------------------
// LayerNorm (norm.rs:55-95): y = (x - mean) * invstd * w + b with the biased
// variance; mean and invstd are saved per row as f32 (adjoint lib.rs:78-85).
// ---------------------------------------------------------------------------

// 8 elements held as their raw 16-byte words (one uint4 for bf16, two for f32), so a
// row can be fetched one iteration ahead at half (bf16) the registers of floats.
template <typename T>
struct Raw8 {
  uint4 u[sizeof(T) / 2];
};
template <typename T>
__device__ __forceinline__ void ldraw(const T* p, Raw8<T>& r) {
#pragma unroll
  for (int k = 0; k < (int)(sizeof(T) / 2); ++k) r.u[k] = reinterpret_cast<const uint4*>(p)[k];
}
__device__ __forceinline__ void unraw(const Raw8<__nv_bfloat16>& r, float (&v)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r.u[0]);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}
__device__ __forceinline__ void unraw(const Raw8<float>& r, float (&v)[8]) {
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    v[4 * k] = __uint_as_float(r.u[k].x);
    v[4 * k + 1] = __uint_as_float(r.u[k].y);
    v[4 * k + 2] = __uint_as_float(r.u[k].z);
    v[4 * k + 3] = __uint_as_float(r.u[k].w);
  }
}

// Two block-wide sums at once for blockDim.x == 256; `red` holds 16 floats.
__device__ __forceinline__ void block_sum2_256(float& a, float& b, float* red) {
  a = warp_sum(a);
  b = warp_sum(b);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) {
    red[w] = a;
    red[8 + w] = b;
  }
  __syncthreads();
  a = warp_sum(l < 8 ? red[l] : 0.0f);
  b = warp_sum(l < 8 ? red[8 + l] : 0.0f);
}

// One CTA of 256 threads per row (norm.rs:5-9 `rowwise`), grid-stride over rows.
// The row stays in registers from the load to the store: the variance is taken
// about the mean (two reductions, no E[x^2] - E[x]^2 cancellation) at one HBM
// read and one write per element.  The next row's words are fetched before this
// row's reductions, so each CTA keeps a row of loads in flight while it waits at
// the barriers.  dim % 8 == 0, dim <= 256 * 8 * VEC and 16-byte aligned pointers
// (the host picks k_layernorm_fwd_any otherwise).
// LayerNorm forward with WPR warps per bf16 row (norm.rs:56-73), the layout and loads of
// k_rmsnorm_fwd_warp: the row stays in registers as bf16 and is unpacked for each of the
// three passes (sum; sum of squared deviations from the mean; output), each reduction a
// warp shuffle plus, for two warps per row, one exchange through shared memory.  Same
// arithmetic as k_layernorm_fwd (biased variance about the mean).
template <int NCH, int WPR>
__global__ void __launch_bounds__(256, 2) k_layernorm_fwd_warp(__nv_bfloat16* __restrict__ y, float* __restrict__ mean,
                                                               float* __restrict__ invstd,
                                                               const __nv_bfloat16* __restrict__ x,
                                                               const __nv_bfloat16* __restrict__ w,
                                                               const __nv_bfloat16* __restrict__ b, long long rows,
                                                               int dim, float eps) {
  static_assert(WPR == 1 || WPR == 2, "one or two warps per row");
  __shared__ float part_s[8], part_q[8];
  const int lane = (int)(threadIdx.x & 31u), warp = (int)(threadIdx.x >> 5);
  const int slot = warp / WPR, sub = warp % WPR;
  constexpr int SLOTS = 8 / WPR;
  const long long ns = (long long)gridDim.x * SLOTS;
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  const uint4* bv = reinterpret_cast<const uint4*>(b);
  for (long long r = (long long)blockIdx.x * SLOTS + slot; r < rows; r += ns) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + r * dim);
    uint4 u[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) u[c] = __ldcs(xr + (c * WPR + sub) * 32 + lane);
    float s = 0.0f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[c]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]);
        s += f.x;
        s += f.y;
      }
    }
    s = warp_sum(s);
    if constexpr (WPR == 2) {
      if (lane == 0) part_s[warp] = s;
      named_bar_sync(1 + slot, 64);
      s = part_s[2 * slot] + part_s[2 * slot + 1];
    }
    const float mu = s / (float)dim;
    float ss = 0.0f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[c]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]);
        const float d0 = f.x - mu, d1 = f.y - mu;
        ss = fmaf(d0, d0, ss);
        ss = fmaf(d1, d1, ss);
      }
    }
    ss = warp_sum(ss);
    if constexpr (WPR == 2) {
      if (lane == 0) part_q[warp] = ss;
      named_bar_sync(1 + slot, 64);  // also: both warps have read part_s before the next row's
      ss = part_q[2 * slot] + part_q[2 * slot + 1];
    }
    const float is = 1.0f / sqrtf(ss / (float)dim + eps);
    if (lane == 0 && sub == 0) {
      mean[r] = mu;
      invstd[r] = is;
    }
    uint4* yr = reinterpret_cast<uint4*>(y + r * dim);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int v = (c * WPR + sub) * 32 + lane;
      const uint4 gu = __ldg(wv + v), bu = __ldg(bv + v);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[c]);
      const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&gu);
      const __nv_bfloat162* bh = reinterpret_cast<const __nv_bfloat162*>(&bu);
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]), g = __bfloat1622float2(gh[k]), c2 = __bfloat1622float2(bh[k]);
        o[k] = pack_bf16x2(fmaf((f.x - mu) * is, g.x, c2.x), fmaf((f.y - mu) * is, g.y, c2.y));
      }
      __stcs(yr + v, make_uint4(o[0], o[1], o[2], o[3]));
    }
  }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(256) k_layernorm_fwd(T* __restrict__ y, float* __restrict__ mean,
                                                       float* __restrict__ invstd, const T* __restrict__ x,
                                                       const T* __restrict__ w, const T* __restrict__ b,
                                                       long long rows, int dim, float eps) {
  __shared__ float red[8];
  const int nvec = dim / 8;
  Raw8<T> nx[VEC];
  long long r = blockIdx.x;
  if (r < rows) {
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi < nvec) ldraw(x + r * dim + vi * 8, nx[i]);
    }
  }
  for (; r < rows; r += gridDim.x) {
    float v[VEC][8];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi < nvec) {
        unraw(nx[i], v[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) s += v[i][j];
      }
    }
    const long long rn = r + gridDim.x;
    if (rn < rows) {
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const int vi = threadIdx.x + i * 256;
        if (vi < nvec) ldraw(x + rn * dim + vi * 8, nx[i]);
      }
    }
    const float mu = block_sum_256(s, red) / (float)dim;
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi < nvec) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[i][j] -= mu;
          ss = fmaf(v[i][j], v[i][j], ss);
        }
      }
    }
    const float is = 1.0f / sqrtf(block_sum_256(ss, red) / (float)dim + eps);
    if (threadIdx.x == 0) {
      mean[r] = mu;
      invstd[r] = is;
    }
    T* yr = y + r * dim;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi < nvec) {
        float g[8], c[8], o[8];
        load8(w + vi * 8, g);
        load8(b + vi * 8, c);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = fmaf(v[i][j] * is, g[j], c[j]);
        store8(yr + vi * 8, o);
      }
    }
  }
}

// Any dim and alignment: three passes over the row (the second and third from L1/L2).
template <typename T>
__global__ void __launch_bounds__(256) k_layernorm_fwd_any(T* __restrict__ y, float* __restrict__ mean,
                                                           float* __restrict__ invstd, const T* __restrict__ x,
                                                           const T* __restrict__ w, const T* __restrict__ b,
                                                           long long rows, int dim, float eps) {
  __shared__ float red[8];
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* xr = x + r * dim;
    float s = 0.0f;
    for (int e = threadIdx.x; e < dim; e += 256) s += ldf(xr + e);
    const float mu = block_sum_256(s, red) / (float)dim;
    float ss = 0.0f;
    for (int e = threadIdx.x; e < dim; e += 256) {
      const float t = ldf(xr + e) - mu;
      ss = fmaf(t, t, ss);
    }
    const float is = 1.0f / sqrtf(block_sum_256(ss, red) / (float)dim + eps);
    if (threadIdx.x == 0) {
      mean[r] = mu;
      invstd[r] = is;
    }
    for (int e = threadIdx.x; e < dim; e += 256)
      stf(y + r * dim + e, fmaf((ldf(xr + e) - mu) * is, ldf(w + e), ldf(b + e)));
  }
}

// Backward, with xh = (x - mean) invstd and e = w dy:
//   dx = invstd (e - mean_d e - xh mean_d(e xh))
// and per-CTA partial column sums of dy xh (dweight) and dy (dbias) into
// part_w / part_b [gridDim.x, dim] (f32; either may be null), summed by k_colsum.
// `vec`: dim % 8 == 0 and every pointer 16-byte aligned.
template <typename T>
__global__ void __launch_bounds__(256) k_layernorm_bwd(T* __restrict__ dx, float* __restrict__ part_w,
                                                       float* __restrict__ part_b, const T* __restrict__ dy,
                                                       const T* __restrict__ x, const float* __restrict__ mean,
                                                       const float* __restrict__ invstd, const T* __restrict__ w,
                                                       long long rows, int dim, bool vec) {
  __shared__ float red[16];
  float* pw = part_w ? part_w + (long long)blockIdx.x * dim : nullptr;
  float* pb = part_b ? part_b + (long long)blockIdx.x * dim : nullptr;
  for (int e = threadIdx.x; e < dim; e += 256) {
    if (pw) pw[e] = 0.0f;
    if (pb) pb[e] = 0.0f;
  }
  __syncthreads();
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* xr = x + r * dim;
    const T* dyr = dy + r * dim;
    const float mu = mean[r], is = invstd[r];
    float sg = 0.0f, sgx = 0.0f;
    if (vec) {
      for (int vi = threadIdx.x; vi < dim / 8; vi += 256) {
        float a[8], d[8], g[8];
        load8(xr + vi * 8, a);
        load8(dyr + vi * 8, d);
        load8(w + vi * 8, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float e = g[j] * d[j];
          sg += e;
          sgx = fmaf(e, (a[j] - mu) * is, sgx);
        }
      }
    } else {
      for (int i = threadIdx.x; i < dim; i += 256) {
        const float e = ldf(w + i) * ldf(dyr + i);
        sg += e;
        sgx = fmaf(e, (ldf(xr + i) - mu) * is, sgx);
      }
    }
    block_sum2_256(sg, sgx, red);
    const float mg = sg / (float)dim, mgx = sgx / (float)dim;
    T* dxr = dx + r * dim;
    if (vec) {
      for (int vi = threadIdx.x; vi < dim / 8; vi += 256) {
        float a[8], d[8], g[8], o[8];
        load8(xr + vi * 8, a);
        load8(dyr + vi * 8, d);
        load8(w + vi * 8, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = (a[j] - mu) * is;
          o[j] = is * (g[j] * d[j] - mg - xh * mgx);
          if (pw) pw[vi * 8 + j] += d[j] * xh;
          if (pb) pb[vi * 8 + j] += d[j];
        }
        store8(dxr + vi * 8, o);
      }
    } else {
      for (int i = threadIdx.x; i < dim; i += 256) {
        const float a = ldf(xr + i), d = ldf(dyr + i);
        const float xh = (a - mu) * is;
        stf(dxr + i, is * (ldf(w + i) * d - mg - xh * mgx));
        if (pw) pw[i] += d * xh;
        if (pb) pb[i] += d;
      }
    }
  }
}

// Backward for dim % 8 == 0, dim <= 256 * 8 * VEC and 16-byte aligned pointers
// (part_w / part_b included).  Same arithmetic as k_layernorm_bwd, but a thread
// owns the same 8 * VEC columns of every row its CTA visits, so the row (x and dy,
// read once from HBM) and the dweight / dbias partial sums stay in registers, and
// each CTA writes its two partial rows once, at the end.  The next row's x and dy
// words are fetched before this row's reduction; the weight is re-read per row
// (an L1 hit) to leave registers for them.
template <typename T, int VEC>
__global__ void __launch_bounds__(256, VEC <= 2 ? 2 : 1)
    k_layernorm_bwd_rows(T* __restrict__ dx, float* __restrict__ part_w, float* __restrict__ part_b,
                         const T* __restrict__ dy, const T* __restrict__ x, const float* __restrict__ mean,
                         const float* __restrict__ invstd, const T* __restrict__ w, long long rows, int dim) {
  __shared__ float red[16];
  const int nvec = dim / 8;
  float aw[VEC][8], ab[VEC][8];
#pragma unroll
  for (int i = 0; i < VEC; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) aw[i][j] = ab[i][j] = 0.0f;
  Raw8<T> nx[VEC], nd[VEC];
  float nmu = 0.0f, nis = 0.0f;
  long long r = blockIdx.x;
  if (r < rows) {
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi < nvec) {
        ldraw(x + r * dim + vi * 8, nx[i]);
        ldraw(dy + r * dim + vi * 8, nd[i]);
      }
    }
    nmu = mean[r];
    nis = invstd[r];
  }
  for (; r < rows; r += gridDim.x) {
    const float mu = nmu, is = nis;
    float xh[VEC][8], d[VEC][8];
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi < nvec) {
        unraw(nx[i], xh[i]);
        unraw(nd[i], d[i]);
      }
    }
    const long long rn = r + gridDim.x;
    if (rn < rows) {
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const int vi = threadIdx.x + i * 256;
        if (vi < nvec) {
          ldraw(x + rn * dim + vi * 8, nx[i]);
          ldraw(dy + rn * dim + vi * 8, nd[i]);
        }
      }
      nmu = mean[rn];
      nis = invstd[rn];
    }
    float sg = 0.0f, sgx = 0.0f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi < nvec) {
        float g[8];
        load8(w + vi * 8, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xh[i][j] = (xh[i][j] - mu) * is;
          const float e = g[j] * d[i][j];
          sg += e;
          sgx = fmaf(e, xh[i][j], sgx);
        }
      }
    }
    block_sum2_256(sg, sgx, red);
    const float mg = sg / (float)dim, mgx = sgx / (float)dim;
    T* dxr = dx + r * dim;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi < nvec) {
        float g[8], o[8];
        load8(w + vi * 8, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          o[j] = is * (g[j] * d[i][j] - mg - xh[i][j] * mgx);
          aw[i][j] = fmaf(d[i][j], xh[i][j], aw[i][j]);
          ab[i][j] += d[i][j];
        }
        store8(dxr + vi * 8, o);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int vi = threadIdx.x + i * 256;
    if (vi < nvec) {
      if (part_w) store8(part_w + (long long)blockIdx.x * dim + vi * 8, aw[i]);
      if (part_b) store8(part_b + (long long)blockIdx.x * dim + vi * 8, ab[i]);
    }
  }
}

// out{0,1}[d] = sum_i part{0,1}[i, d] for the LayerNorm parameter gradients, both in
// one launch (blockIdx.y picks the pair; a null `out` skips it).  A CTA owns 32
// columns and its 8 warps split the partial rows, so each thread issues
// nparts / 8 coalesced loads instead of nparts.
template <typename T>
__global__ void __launch_bounds__(256) k_colsum_split2(T* __restrict__ out0, const float* __restrict__ part0,
                                                       T* __restrict__ out1, const float* __restrict__ part1,
                                                       int nparts, int dim) {
  __shared__ float red[8][33];
  T* out = blockIdx.y ? out1 : out0;
  const float* part = blockIdx.y ? part1 : part0;
  if (out == nullptr) return;  // uniform across the CTA
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int d = blockIdx.x * 32 + lane;
  float s = 0.0f;
  if (d < dim)
    for (int i = wp; i < nparts; i += 8) s += part[(long long)i * dim + d];
  red[wp][lane] = s;
  __syncthreads();
  if (wp == 0 && d < dim) {
    float t = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k][lane];
    stf(out + d, t);
  }
}

// RMSNorm backward for dim % 8 == 0, dim <= 256 * 8 * VEC and 16-byte aligned
// pointers (part included): the arithmetic of k_rmsnorm_bwd with the row layout of
// k_layernorm_bwd_rows (row and dweight partials in registers, next row fetched
// before the reduction, one partial row per CTA written at the end).
template <typename T, int VEC>
__global__ void __launch_bounds__(256, VEC <= 2 ? 2 : 1)
    k_rmsnorm_bwd_rows(T* __restrict__ dx, float* __restrict__ part, const T* __restrict__ dy,
                       const T* __restrict__ x, const float* __restrict__ rms, const T* __restrict__ w,
                       long long rows, int dim) {
  __shared__ float red[8];
  const int nvec = dim / 8;
  float aw[VEC][8];
#pragma unroll
  for (int i = 0; i < VEC; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) aw[i][j] = 0.0f;
  Raw8<T> nx[VEC], nd[VEC];
  float nr = 1.0f;
  long long r = blockIdx.x;
  if (r < rows) {
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi < nvec) {
        ldraw(x + r * dim + vi * 8, nx[i]);
        ldraw(dy + r * dim + vi * 8, nd[i]);
      }
    }
    nr = rms[r];
  }
  for (; r < rows; r += gridDim.x) {
    const float inv = 1.0f / nr;
    float a[VEC][8], d[VEC][8];
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi < nvec) {
        unraw(nx[i], a[i]);
        unraw(nd[i], d[i]);
      }
    }
    const long long rn = r + gridDim.x;
    if (rn < rows) {
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const int vi = threadIdx.x + i * 256;
        if (vi < nvec) {
          ldraw(x + rn * dim + vi * 8, nx[i]);
          ldraw(dy + rn * dim + vi * 8, nd[i]);
        }
      }
      nr = rms[rn];
    }
    float dot = 0.0f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi < nvec) {
        float g[8];
        load8(w + vi * 8, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) dot = fmaf(g[j] * d[i][j], a[i][j], dot);
      }
    }
    dot = block_sum_256(dot, red);
    const float c = dot * inv * inv * inv / (float)dim;
    T* dxr = dx + r * dim;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi < nvec) {
        float g[8], o[8];
        load8(w + vi * 8, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          o[j] = g[j] * d[i][j] * inv - a[i][j] * c;
          aw[i][j] += d[i][j] * a[i][j] * inv;
        }
        store8(dxr + vi * 8, o);
      }
    }
  }
  if (part) {
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int vi = threadIdx.x + i * 256;
      if (vi < nvec) store8(part + (long long)blockIdx.x * dim + vi * 8, aw[i]);
    }
  }
}

// RMSNorm backward with WPR warps per bf16 row (norm.rs:33-50), the row layout of
// k_rmsnorm_fwd_warp: a lane holds 8 x NCH columns of the row (dim = 256 x NCH x WPR),
// loaded with 16-byte streaming loads, so every resident warp has its row's x and dy in
// flight and no CTA-wide barrier holds the other rows back.  The arithmetic is
// k_rmsnorm_bwd_rows' (dot = sum w dy x; dx = w dy / rms - x dot / (rms^3 dim)); each lane
// keeps its weight columns and its dweight partials (sum dy x / rms) in registers across
// the rows it visits, and at the end the CTA's row slots add their partials in shared
// memory in slot order and write one partial row per CTA for k_colsum_split2.
template <int NCH, int WPR>
__global__ void __launch_bounds__(256, 2) k_rmsnorm_bwd_warp(__nv_bfloat16* __restrict__ dx, float* __restrict__ part,
                                                             const __nv_bfloat16* __restrict__ dy,
                                                             const __nv_bfloat16* __restrict__ x,
                                                             const float* __restrict__ rms,
                                                             const __nv_bfloat16* __restrict__ w, long long rows,
                                                             int dim) {
  static_assert(WPR == 1 || WPR == 2 || WPR == 4, "one, two or four warps per row");
  static_assert(NCH >= 1 && NCH <= 4, "at most 32 columns per lane");
  constexpr int SLOTS = 8 / WPR;
  __shared__ float dots[8];
  __shared__ __align__(16) float acc[256 * 4 * 4];  // the CTA's dweight partial row (dim <= 4096)
  const int lane = (int)(threadIdx.x & 31u), warp = (int)(threadIdx.x >> 5);
  const int slot = warp / WPR, sub = warp % WPR;
  const long long ns = (long long)gridDim.x * SLOTS;
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  uint4 gu[NCH];
  float aw[NCH][8];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    gu[c] = __ldg(wv + (c * WPR + sub) * 32 + lane);
#pragma unroll
    for (int j = 0; j < 8; ++j) aw[c][j] = 0.0f;
  }
  for (long long r = (long long)blockIdx.x * SLOTS + slot; r < rows; r += ns) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + r * dim);
    const uint4* dr = reinterpret_cast<const uint4*>(dy + r * dim);
    uint4 ux[NCH], ud[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      ux[c] = __ldcs(xr + (c * WPR + sub) * 32 + lane);
      ud[c] = __ldcs(dr + (c * WPR + sub) * 32 + lane);
    }
    const float inv = 1.0f / __ldg(rms + r);
    float dot = 0.0f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const __nv_bfloat162* hx = reinterpret_cast<const __nv_bfloat162*>(&ux[c]);
      const __nv_bfloat162* hd = reinterpret_cast<const __nv_bfloat162*>(&ud[c]);
      const __nv_bfloat162* hg = reinterpret_cast<const __nv_bfloat162*>(&gu[c]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a = __bfloat1622float2(hx[j]), d = __bfloat1622float2(hd[j]), g = __bfloat1622float2(hg[j]);
        dot = fmaf(g.x * d.x, a.x, dot);
        dot = fmaf(g.y * d.y, a.y, dot);
      }
    }
    dot = warp_sum(dot);
    if constexpr (WPR > 1) {
      if (lane == 0) dots[warp] = dot;
      named_bar_sync(1 + slot, 32 * WPR);
      dot = 0.0f;
#pragma unroll
      for (int i = 0; i < WPR; ++i) dot += dots[slot * WPR + i];
      named_bar_sync(1 + slot, 32 * WPR);  // every warp of the slot has read the partials
    }
    // the rows stay packed across the reduction: the unpacked floats are formed again below
    // rather than held (64 more registers at NCH = 4, which spilled)
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      asm volatile("" : "+r"(ux[c].x), "+r"(ux[c].y), "+r"(ux[c].z), "+r"(ux[c].w));
      asm volatile("" : "+r"(ud[c].x), "+r"(ud[c].y), "+r"(ud[c].z), "+r"(ud[c].w));
      asm volatile("" : "+r"(gu[c].x), "+r"(gu[c].y), "+r"(gu[c].z), "+r"(gu[c].w));
    }
    const float cc = dot * inv * inv * inv / (float)dim;
    uint4* xo = reinterpret_cast<uint4*>(dx + r * dim);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const __nv_bfloat162* hx = reinterpret_cast<const __nv_bfloat162*>(&ux[c]);
      const __nv_bfloat162* hd = reinterpret_cast<const __nv_bfloat162*>(&ud[c]);
      const __nv_bfloat162* hg = reinterpret_cast<const __nv_bfloat162*>(&gu[c]);
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a = __bfloat1622float2(hx[j]), d = __bfloat1622float2(hd[j]), g = __bfloat1622float2(hg[j]);
        o[j] = pack_bf16x2(g.x * d.x * inv - a.x * cc, g.y * d.y * inv - a.y * cc);
        aw[c][2 * j] += d.x * a.x * inv;
        aw[c][2 * j + 1] += d.y * a.y * inv;
      }
      __stcs(xo + (c * WPR + sub) * 32 + lane, make_uint4(o[0], o[1], o[2], o[3]));
    }
  }
  if (part == nullptr) return;  // uniform over the grid
#pragma unroll 1
  for (int s = 0; s < SLOTS; ++s) {
    if (slot == s) {
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        float4* p4 = reinterpret_cast<float4*>(acc + ((c * WPR + sub) * 32 + lane) * 8);
        float4 lo = make_float4(aw[c][0], aw[c][1], aw[c][2], aw[c][3]);
        float4 hi = make_float4(aw[c][4], aw[c][5], aw[c][6], aw[c][7]);
        if (s > 0) {
          const float4 plo = p4[0], phi = p4[1];
          lo = make_float4(plo.x + lo.x, plo.y + lo.y, plo.z + lo.z, plo.w + lo.w);
          hi = make_float4(phi.x + hi.x, phi.y + hi.y, phi.z + hi.z, phi.w + hi.w);
        }
        p4[0] = lo;
        p4[1] = hi;
      }
    }
    __syncthreads();
  }
  float4* prow = reinterpret_cast<float4*>(part + (long long)blockIdx.x * dim);
  const float4* a4 = reinterpret_cast<const float4*>(acc);
  for (int i = (int)threadIdx.x; i < dim / 4; i += 256) prow[i] = a4[i];
}

// ---------------------------------------------------------------------------
// SwiGLU elementwise pieces (mlp.rs:12-52); silu(z) = z * sigmoid(z)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float sigmoid_f(float z) { return 1.0f / (1.0f + expf(-z)); }

// h = silu(gate) * up
template <typename T>
__global__ void k_swiglu_h(T* __restrict__ h, const T* __restrict__ gate, const T* __restrict__ up, long long n) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float g = ldf(gate + i), u = ldf(up + i);
    stf(h + i, g * sigmoid_f(g) * u);
  }
}

// In place: gate <- dgate = dh * up * s * (1 + g (1 - s)),  up <- dup = dh * silu(g),  s = sigmoid(g).
// Optionally also writes h = silu(g) * up first (for dWd).
template <typename T>
__global__ void k_swiglu_bwd_elem(T* __restrict__ gate, T* __restrict__ up, const T* __restrict__ dh, long long n) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float g = ldf(gate + i), u = ldf(up + i), d = ldf(dh + i);
    const float s = sigmoid_f(g);
    stf(gate + i, d * u * s * (1.0f + g * (1.0f - s)));
    stf(up + i, d * g * s);
  }
}

}  // namespace beacon
