// Append-time codec shared by the encode kernels and the fused decode step: polar keys and
// grouped int8 values of one 64-token page, written in the kernel page layout.
//
// Numerics follow the reference encoder op by op (rfsn_v11/quant/polar/encoder.py:24-130,
// rfsn_v11/quant/v_quant/encoder.py:16-30): every float16 op rounds once to float16 (an
// fp32 op of two fp16 operands followed by round-to-nearest is the correctly rounded fp16
// result for + - * / sqrt), transcendentals are evaluated in float64 and rounded to float32
// (a correctly rounded float32 atan2 / log), and the multiply by 2^bits-1 plus the
// half-to-even round happen in float32 because the encoder's mx.where(..., mx.array(0.0), ...)
// promotes the normalised angle to float32.
#pragma once

#include "tp_common.cuh"

namespace tp {

// Largest page block of any supported format: float16 radii, 64 code bytes per token.
constexpr int kMaxUnitBytes = kUnit * 128 + kVCodesUnit + kUnit * 64 + kVScalesUnit;
constexpr int kMaxPageBytes = 2 * kMaxUnitBytes;

// ----------------------------------------------------------------------------- codec math
// float32 (cos, sin) of the decoder angle of a `bits`-bit code: code / (2^bits - 1) * 2pi - pi
// with each op rounded to float32 (rfsn_v11/quant/polar/decoder.py:36-56), cos and sin
// evaluated in float64 and rounded to float32.
__device__ __forceinline__ float2 cos_sin_of_code(int code, int bits) {
  const int lm1 = (1 << bits) - 1;
  const float norm = __fdiv_rn(float(code), float(lm1));
  const float ang = __fsub_rn(__fmul_rn(norm, 6.28318530717958647692f), 3.14159265358979323846f);
  return make_float2(d2f(cos(double(ang))), d2f(sin(double(ang))));
}

struct PairCode {
  __half r;     // float16 radius
  float norm;   // normalised angle in [0, 1] (float32, the promoted value)
};

// encoder.py:33 and :46-51 for float16 input.
__device__ __forceinline__ PairCode polar_pair(__half x, __half y) {
  const float xf = __half2float(x), yf = __half2float(y);
  const __half xx = __float2half_rn(__fmul_rn(xf, xf));
  const __half yy = __float2half_rn(__fmul_rn(yf, yf));
  const __half s = __float2half_rn(__fadd_rn(__half2float(xx), __half2float(yy)));
  PairCode pc;
  pc.r = __float2half_rn(__fsqrt_rn(__half2float(s)));
  const __half a = __float2half_rn(d2f(atan2(double(yf), double(xf))));
  const __half sh = __float2half_rn(__fadd_rn(__half2float(a), 3.140625f));   // fp16(pi)
  const __half n = __float2half_rn(__fdiv_rn(__half2float(sh), 6.28125f));    // fp16(2pi)
  // clip(0, 1); the "> fp16(1 - 1e-6) = 1.0 -> 0" branch cannot fire after the clip.
  pc.norm = fminf(fmaxf(__half2float(n), 0.0f), 1.0f);
  return pc;
}

// The same for float32 input (all ops in float32, radius stored as float16).
__device__ __forceinline__ PairCode polar_pair(float x, float y) {
  const float s = __fadd_rn(__fmul_rn(x, x), __fmul_rn(y, y));
  PairCode pc;
  pc.r = __float2half_rn(__fsqrt_rn(s));
  const float a = d2f(atan2(double(y), double(x)));
  const float sh = __fadd_rn(a, 3.14159265358979323846f);
  float n = __fdiv_rn(sh, 6.28318530717958647692f);
  n = fminf(fmaxf(n, 0.0f), 1.0f);
  if (n > float(1.0 - 1e-6)) n = 0.0f;
  pc.norm = n;
  return pc;
}

__device__ __forceinline__ uint8_t angle_code(float norm, int bits) {
  const float lm1 = float((1 << bits) - 1);
  const float c = rintf(__fmul_rn(norm, lm1));
  return static_cast<uint8_t>(fminf(fmaxf(c, 0.0f), lm1));
}

// log(max(r, fp16(1e-6))) rounded to float16 then widened (encoder.py:37).
__device__ __forceinline__ float log_radius(__half r) {
  const float floor16 = 1.0132789611816406e-06f;  // float16(1e-6) = 17 * 2^-24
  const float rf = fmaxf(__half2float(r), floor16);
  return __half2float(__float2half_rn(d2f(log(double(rf)))));
}

// v_quant/encoder.py:22-25 for one group of 32 values.
__device__ __forceinline__ __half v_group_scale(float max_abs, bool f16_input) {
  (void)f16_input;  // fp16: correctly rounded fp16 division; fp32: fp32 division then fp16.
  __half s = __float2half_rn(__fdiv_rn(max_abs, 127.0f));
  if (__half2float(s) == 0.0f) s = __ushort_as_half(1678);  // float16(1e-4)
  return s;
}

__device__ __forceinline__ int8_t v_code(float v, float scale, bool f16_input) {
  float q = __fdiv_rn(v, scale);
  if (f16_input) q = __half2float(__float2half_rn(q));
  q = rintf(q);
  return static_cast<int8_t>(fminf(fmaxf(q, -128.0f), 127.0f));
}

template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }

// Encode one 64-token page of one head into the page block s_page (shared memory, laid out
// as in the pool) and its radius scale into *s_radius_scale (int8 radii only).  256 threads:
// thread (token l = tid/4, quarter c = tid%4) owns pairs [16c, 16c+16) and V group c of
// token l.  Ends with a barrier, so the caller may copy the block out.
template <typename T>
__device__ void encode_page(const T* k_rows, const T* v_rows, int64_t row_stride, const PoolArgs& P, uint8_t* s_page,
                            __half* s_radius_scale, uint8_t* s_codes, float* s_red, const T* k_last = nullptr,
                            const T* v_last = nullptr) {
  const int tid = threadIdx.x;
  const int l = tid >> 2, c = tid & 3;
  const bool f16_in = sizeof(T) == 2;
  const bool last = k_last != nullptr && l == kPage - 1;  // token 63 read from its own row
  const T* kr = (last ? k_last : k_rows + l * row_stride) + 32 * c;
  float logr[16];
  __half rad[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int j = 16 * c + i;
    const PairCode pc = polar_pair(kr[2 * i], kr[2 * i + 1]);
    rad[i] = pc.r;
    s_codes[l * kPairs + j] = angle_code(pc.norm, j < P.l1_pairs ? P.l1_bits : P.deep_bits);
    if (P.int8_radii) logr[i] = log_radius(pc.r);
  }
  if (!P.int8_radii) {
    // Chunks 2c and 2c+1 of row l, stored at their swizzled positions.
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        w[i] = uint32_t(__half_as_ushort(rad[8 * h + 2 * i])) | (uint32_t(__half_as_ushort(rad[8 * h + 2 * i + 1])) << 16);
      *reinterpret_cast<uint4*>(radius_f16_at(P, s_page, l, 16 * c + 8 * h)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
    // encoder.py:38-45: one scale per (head, block) = max|log r| / 127.
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(logr[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((tid & 31) == 0) s_red[tid >> 5] = m;
    __syncthreads();
    m = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, s_red[w]);
    const float ls = (m == 0.0f) ? 1e-6f : m;
    const __half sc = __float2half_rn(__fdiv_rn(ls, 127.0f));
    const float scf = __half2float(sc);
    int8_t* rr = radius_i8_at(P, s_page, l, 16 * c);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float q = rintf(__fdiv_rn(logr[i], scf));
      rr[i] = static_cast<int8_t>(fminf(fmaxf(q, -128.0f), 127.0f));
    }
    if (tid == 0) *s_radius_scale = sc;
  }
  // Values: group c of token l.
  {
    const T* vr = (last ? v_last : v_rows + l * row_stride) + 32 * c;
    float vals[32];
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      vals[i] = to_f(vr[i]);
      mx = fmaxf(mx, fabsf(vals[i]));
    }
    const __half sc = v_group_scale(mx, f16_in);
    const float scf = __half2float(sc);
#pragma unroll
    for (int i = 0; i < 32; ++i) *vcode_at(P, s_page, l, 32 * c + i) = uint8_t(v_code(vals[i], scf, f16_in)) ^ 0x80u;
    *vscale_at(P, s_page, l, c) = sc;
  }
  __syncthreads();
  // Pack the angle codes row by row (encoder.py:56-75, :100-130): level-1 bytes, then deep.
  for (int i = tid; i < kPage * P.code_row; i += blockDim.x) {
    const int tok = i / P.code_row, byte = i - tok * P.code_row;
    const bool is_l1 = byte < P.l1_row;
    const int bb = is_l1 ? byte : byte - P.l1_row;
    const int bits = is_l1 ? P.l1_bits : P.deep_bits;
    const int n = is_l1 ? P.l1_pairs : kPairs - P.l1_pairs;
    const uint8_t* codes = s_codes + tok * kPairs + (is_l1 ? 0 : P.l1_pairs);
    uint8_t out;
    if (bits == 8) {
      out = codes[bb];
    } else {
      const int per = 8 / bits, mask = (1 << bits) - 1;
      out = 0;
      for (int q = 0; q < per; ++q) {
        const int idx = bb * per + q;
        if (idx < n) out |= uint8_t((codes[idx] & mask) << (q * bits));
      }
    }
    codes_at(P, s_page, tok)[byte] = out;
  }
  __syncthreads();
}

// Copy an encoded page block from shared memory to pool page `page` of head h (all threads).
__device__ __forceinline__ void store_page_block(const PoolArgs& P, const uint8_t* s_page, __half radius_scale, int h,
                                                 int page) {
  uint4* dst = reinterpret_cast<uint4*>(P.page(h, page));
  for (int i = threadIdx.x; i < P.page_bytes / 16; i += blockDim.x) dst[i] = reinterpret_cast<const uint4*>(s_page)[i];
  if (threadIdx.x == 0 && P.int8_radii) *P.radii_scale(h, page) = radius_scale;
}

}  // namespace tp
