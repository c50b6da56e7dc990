// Append-time encoding: polar keys + grouped int8 values written straight into the device
// page pool, and the tail-append kernel that keeps the cache state on the device.
//
// Numerics follow the reference encoder op by op (rfsn_v11/quant/polar/encoder.py:24-130,
// rfsn_v11/quant/v_quant/encoder.py:16-30): every float16 op rounds once to float16 (an
// fp32 op of two fp16 operands followed by round-to-nearest is the correctly rounded fp16
// result for + - * / sqrt), transcendentals are evaluated in float64 and rounded to float32
// (a correctly rounded float32 atan2 / log), and the multiply by 2^bits-1 plus the
// half-to-even round happen in float32 because the encoder's mx.where(..., mx.array(0.0), ...)
// promotes the normalised angle to float32.
#include <cstdio>
#include <mutex>
#include <string>

#include "tp_common.cuh"

namespace tp {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TP_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return TP_OK;
}

int make_layout(const tp_format& f, Layout* out) {
  if (f.l1_bits != 4 && f.l1_bits != 8)
    return fail(TP_ERR_UNSUPPORTED, "unsupported k_angle_bits_level1: " + std::to_string(f.l1_bits));
  if (f.deep_bits != 2 && f.deep_bits != 4 && f.deep_bits != 8)
    return fail(TP_ERR_UNSUPPORTED, "unsupported k_angle_bits_deep: " + std::to_string(f.deep_bits));
  if (f.split_dim < 0 || f.split_dim > kD || (f.split_dim & 1))
    return fail(TP_ERR_INVALID, "split_dim must be even and within [0, head_dim]");
  Layout L;
  L.l1_pairs = f.split_dim / 2;
  L.deep_pairs = kPairs - L.l1_pairs;
  L.l1_row = f.l1_bits == 8 ? L.l1_pairs : (L.l1_pairs + 1) / 2;
  const int per = 8 / f.deep_bits;
  L.deep_row = (L.deep_pairs + per - 1) / per;
  L.radii_row = f.int8_radii ? kPairs : kPairs * 2;
  L.radii_page = int64_t(kPage) * L.radii_row;
  L.l1_page = int64_t(kPage) * L.l1_row;
  L.deep_page = int64_t(kPage) * L.deep_row;
  *out = L;
  return TP_OK;
}

// Pointers of one (head, page) of the pool.
struct PagePtrs {
  uint8_t* radii;
  __half* radii_scale;
  uint8_t* l1;
  uint8_t* deep;
  int8_t* v_codes;
  __half* v_scales;
};

struct PoolArgs {
  uint8_t* radii;
  __half* radii_scales;
  uint8_t* l1;
  uint8_t* deep;
  int8_t* v_codes;
  __half* v_scales;
  int num_kv_heads, page_capacity;
  int l1_bits, deep_bits, split_dim, int8_radii;
  int l1_pairs, l1_row, deep_row, radii_row;

  __device__ PagePtrs page(int h, int p) const {
    const int64_t slot = int64_t(h) * page_capacity + p;
    PagePtrs d;
    d.radii = radii + slot * kPage * radii_row;
    d.radii_scale = int8_radii ? radii_scales + slot : nullptr;
    d.l1 = l1 + slot * kPage * l1_row;
    d.deep = deep + slot * kPage * deep_row;
    d.v_codes = v_codes + slot * kVCodesPage;
    d.v_scales = v_scales + slot * kPage * 4;
    return d;
  }
};

static PoolArgs pool_args(const tp_page_pool& p, const Layout& L) {
  PoolArgs a;
  a.radii = static_cast<uint8_t*>(p.radii);
  a.radii_scales = static_cast<__half*>(p.radii_scales);
  a.l1 = static_cast<uint8_t*>(p.angle_codes_l1);
  a.deep = static_cast<uint8_t*>(p.angle_codes_deep);
  a.v_codes = static_cast<int8_t*>(p.v_codes);
  a.v_scales = static_cast<__half*>(p.v_scales);
  a.num_kv_heads = p.num_kv_heads;
  a.page_capacity = p.page_capacity;
  a.l1_bits = p.fmt.l1_bits;
  a.deep_bits = p.fmt.deep_bits;
  a.split_dim = p.fmt.split_dim;
  a.int8_radii = p.fmt.int8_radii;
  a.l1_pairs = L.l1_pairs;
  a.l1_row = L.l1_row;
  a.deep_row = L.deep_row;
  a.radii_row = L.radii_row;
  return a;
}

int validate_pool(const tp_page_pool* pool, Layout* L, bool keys) {
  if (!pool) return fail(TP_ERR_INVALID, "page pool is NULL");
  int st = make_layout(pool->fmt, L);
  if (st != TP_OK) return st;
  if (pool->num_kv_heads <= 0) return fail(TP_ERR_INVALID, "num_kv_heads must be positive");
  if (pool->page_capacity < 0) return fail(TP_ERR_INVALID, "page_capacity must be >= 0");
  if (pool->page_capacity > 0) {
    if (!pool->v_codes || !pool->v_scales) return fail(TP_ERR_INVALID, "page pool has a NULL value field");
    if (keys) {
      if (!pool->radii) return fail(TP_ERR_INVALID, "page pool has NULL radii");
      if (L->l1_row > 0 && !pool->angle_codes_l1) return fail(TP_ERR_INVALID, "angle_codes_l1 is NULL");
      if (L->deep_row > 0 && !pool->angle_codes_deep) return fail(TP_ERR_INVALID, "angle_codes_deep is NULL");
      if (pool->fmt.int8_radii && !pool->radii_scales) return fail(TP_ERR_INVALID, "int8 radii require radii_scales");
    }
    const void* ptrs[] = {pool->radii, pool->angle_codes_l1, pool->angle_codes_deep, pool->v_codes, pool->v_scales};
    for (const void* q : ptrs)
      if (q && (reinterpret_cast<uintptr_t>(q) & 15))
        return fail(TP_ERR_INVALID, "page pool fields must be 16-byte aligned");
  }
  return TP_OK;
}

// ----------------------------------------------------------------------------- codec math
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

// Encode one 64-token page of one head.  256 threads: thread (token l = tid/4, quarter c = tid%4)
// owns pairs [16c, 16c+16) and V group c of token l.
template <typename T>
__device__ void encode_page(const T* k_rows, const T* v_rows, int64_t row_stride, const PagePtrs& dst,
                            const PoolArgs& P, uint8_t* s_codes, float* s_red, uint8_t* s_v, __half* s_scales) {
  const int tid = threadIdx.x;
  const int l = tid >> 2, c = tid & 3;
  const bool f16_in = sizeof(T) == 2;
  const T* kr = k_rows + l * row_stride + 32 * c;
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
      *reinterpret_cast<uint4*>(dst.radii + radii_f16_offset(l, 16 * c + 8 * h)) = make_uint4(w[0], w[1], w[2], w[3]);
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
    int8_t* rr = reinterpret_cast<int8_t*>(dst.radii) + l * kPairs + 16 * c;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float q = rintf(__fdiv_rn(logr[i], scf));
      rr[i] = static_cast<int8_t>(fminf(fmaxf(q, -128.0f), 127.0f));
    }
    if (tid == 0) *dst.radii_scale = sc;
  }
  // Values: group c of token l.
  {
    const T* vr = v_rows + l * row_stride + 32 * c;
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
    for (int i = 0; i < 32; ++i) s_v[vcode_offset(l, 32 * c + i)] = uint8_t(v_code(vals[i], scf, f16_in)) ^ 0x80u;
    s_scales[vscale_index(l, c)] = sc;
  }
  __syncthreads();
  // Pack the angle codes row by row (encoder.py:56-75, :100-130).
  const int l1_bytes = kPage * P.l1_row, deep_bytes = kPage * P.deep_row;
  for (int i = tid; i < l1_bytes + deep_bytes; i += blockDim.x) {
    const bool is_l1 = i < l1_bytes;
    const int ii = is_l1 ? i : i - l1_bytes;
    const int row = is_l1 ? P.l1_row : P.deep_row;
    const int tok = ii / row, byte = ii % row;
    const int bits = is_l1 ? P.l1_bits : P.deep_bits;
    const int n = is_l1 ? P.l1_pairs : kPairs - P.l1_pairs;
    const uint8_t* codes = s_codes + tok * kPairs + (is_l1 ? 0 : P.l1_pairs);
    uint8_t out;
    if (bits == 8) {
      out = codes[byte];
    } else {
      const int per = 8 / bits, mask = (1 << bits) - 1;
      out = 0;
      for (int q = 0; q < per; ++q) {
        const int idx = byte * per + q;
        if (idx < n) out |= uint8_t((codes[idx] & mask) << (q * bits));
      }
    }
    (is_l1 ? dst.l1 : dst.deep)[ii] = out;
  }
  // Values and scales, staged in the page layout, leave in 16-byte stores.
  for (int i = tid; i < int(kVCodesPage / 16); i += blockDim.x)
    reinterpret_cast<uint4*>(dst.v_codes)[i] = reinterpret_cast<const uint4*>(s_v)[i];
  for (int i = tid; i < int(kVScalesPage / 16); i += blockDim.x)
    reinterpret_cast<uint4*>(dst.v_scales)[i] = reinterpret_cast<const uint4*>(s_scales)[i];
}

template <typename T>
__global__ void __launch_bounds__(256) encode_pages_kernel(PoolArgs P, const T* k, const T* v, int64_t head_stride,
                                                           int64_t token_stride, int64_t src_token0, int dst_page,
                                                           int n_pages, int32_t* d_state) {
  __shared__ uint8_t s_codes[kPage * kPairs];
  __shared__ float s_red[8];
  __shared__ __align__(16) uint8_t s_v[kVCodesPage];
  __shared__ __align__(16) __half s_scales[kPage * 4];
  const int p = blockIdx.x, h = blockIdx.y;
  const int64_t tok0 = src_token0 + int64_t(p) * kPage;
  encode_page<T>(k + h * head_stride + tok0 * token_stride, v + h * head_stride + tok0 * token_stride, token_stride,
                 P.page(h, dst_page + p), P, s_codes, s_red, s_v, s_scales);
  if (d_state) {
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const int total = gridDim.x * gridDim.y;
      if (atomicAdd(&d_state[5], 1) == total - 1) {
        d_state[0] += n_pages;
        d_state[2] += n_pages * kPage;
        d_state[5] = 0;
        __threadfence();
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) append_kernel(PoolArgs P, T* tail_k, T* tail_v, int32_t* d_state, const T* k_new,
                                                     const T* v_new, int64_t head_stride, int64_t token_stride,
                                                     int n_tokens) {
  __shared__ uint8_t s_codes[kPage * kPairs];
  __shared__ float s_red[8];
  __shared__ __align__(16) uint8_t s_v[kVCodesPage];
  __shared__ __align__(16) __half s_scales[kPage * 4];
  const int h = blockIdx.x;
  const int n_pages = d_state[0], tail_len = d_state[1];
  const bool overflow = tail_len < 0 || tail_len + n_tokens > kPage;
  const bool fills = !overflow && tail_len + n_tokens == kPage;
  const bool pool_full = fills && n_pages >= P.page_capacity;
  if (overflow || pool_full) {
    if (h == 0 && threadIdx.x == 0) d_state[4] = overflow ? 1 : 2;
    return;
  }
  T* tk = tail_k + int64_t(h) * kPage * kD;
  T* tv = tail_v + int64_t(h) * kPage * kD;
  for (int i = threadIdx.x; i < n_tokens * kD; i += blockDim.x) {
    const int t = i / kD, d = i % kD;
    const int64_t src = h * head_stride + t * token_stride + d;
    tk[(tail_len + t) * kD + d] = k_new[src];
    tv[(tail_len + t) * kD + d] = v_new[src];
  }
  __syncthreads();
  if (fills) {
    encode_page<T>(tk, tv, kD, P.page(h, n_pages), P, s_codes, s_red, s_v, s_scales);
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&d_state[5], 1) == (int)gridDim.x - 1) {
      d_state[0] = n_pages + (fills ? 1 : 0);
      d_state[1] = fills ? 0 : tail_len + n_tokens;
      d_state[2] += n_tokens;
      d_state[5] = 0;
      __threadfence();
    }
  }
}

}  // namespace tp

using namespace tp;

extern "C" {

const char* tp_last_error(void) { return g_last_error.c_str(); }

int tp_version(void) { return 1; }

int tp_row_bytes(const tp_format* fmt, int32_t* l1_row_bytes, int32_t* deep_row_bytes) {
  if (!fmt) return fail(TP_ERR_INVALID, "format is NULL");
  Layout L;
  int st = make_layout(*fmt, &L);
  if (st != TP_OK) return st;
  if (l1_row_bytes) *l1_row_bytes = L.l1_row;
  if (deep_row_bytes) *deep_row_bytes = L.deep_row;
  return TP_OK;
}

int tp_encode_pages(const tp_page_pool* pool, const void* k, const void* v, int32_t dtype, int64_t head_stride,
                    int64_t token_stride, int64_t src_token0, int32_t n_pages, int32_t dst_page, int32_t* d_state,
                    void* stream) {
  Layout L;
  int st = validate_pool(pool, &L);
  if (st != TP_OK) return st;
  if (n_pages < 0 || dst_page < 0 || int64_t(dst_page) + n_pages > pool->page_capacity)
    return fail(TP_ERR_INVALID, "tp_encode_pages: page range outside the pool");
  if (n_pages == 0) return TP_OK;
  if (!k || !v) return fail(TP_ERR_INVALID, "tp_encode_pages: NULL input");
  PoolArgs P = pool_args(*pool, L);
  dim3 grid(n_pages, pool->num_kv_heads);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == TP_F16)
    encode_pages_kernel<__half><<<grid, 256, 0, s>>>(P, static_cast<const __half*>(k), static_cast<const __half*>(v),
                                                     head_stride, token_stride, src_token0, dst_page, n_pages, d_state);
  else if (dtype == TP_F32)
    encode_pages_kernel<float><<<grid, 256, 0, s>>>(P, static_cast<const float*>(k), static_cast<const float*>(v),
                                                    head_stride, token_stride, src_token0, dst_page, n_pages, d_state);
  else
    return fail(TP_ERR_INVALID, "only float16 and float32 inputs are supported");
  return check_launch("tp_encode_pages");
}

int tp_append(const tp_page_pool* pool, const tp_tail* tail, int32_t* d_state, const void* k_new, const void* v_new,
              int32_t dtype, int64_t head_stride, int64_t token_stride, int32_t n_tokens, void* stream) {
  Layout L;
  int st = validate_pool(pool, &L);
  if (st != TP_OK) return st;
  if (!tail || !tail->k || !tail->v || !d_state || !k_new || !v_new)
    return fail(TP_ERR_INVALID, "tp_append: NULL argument");
  if (n_tokens < 1 || n_tokens > kPage) return fail(TP_ERR_INVALID, "tp_append: n_tokens must be in [1, 64]");
  if (tail->dtype != dtype) return fail(TP_ERR_INVALID, "tp_append: tail dtype differs from input dtype");
  PoolArgs P = pool_args(*pool, L);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = pool->num_kv_heads;
  if (dtype == TP_F16)
    append_kernel<__half><<<grid, 256, 0, s>>>(P, static_cast<__half*>(tail->k), static_cast<__half*>(tail->v), d_state,
                                               static_cast<const __half*>(k_new), static_cast<const __half*>(v_new),
                                               head_stride, token_stride, n_tokens);
  else if (dtype == TP_F32)
    append_kernel<float><<<grid, 256, 0, s>>>(P, static_cast<float*>(tail->k), static_cast<float*>(tail->v), d_state,
                                              static_cast<const float*>(k_new), static_cast<const float*>(v_new),
                                              head_stride, token_stride, n_tokens);
  else
    return fail(TP_ERR_INVALID, "only float16 and float32 inputs are supported");
  return check_launch("tp_append");
}

}  // extern "C"
