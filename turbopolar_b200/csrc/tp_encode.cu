// Append-time encoding: polar keys + grouped int8 values written straight into the device
// page pool (codec in tp_codec.cuh), and the tail-append kernel that keeps the cache state on
// the device.
#include <cstdio>
#include <mutex>
#include <string>

#include "tp_codec.cuh"

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
  L.code_row = L.l1_row + L.deep_row;
  L.radii_row = f.int8_radii ? kPairs : kPairs * 2;
  // Unit: radii | value codes | angle codes | value scales (every size a multiple of 32 bytes).
  L.u_vcodes = kUnit * L.radii_row;
  L.u_codes = L.u_vcodes + kVCodesUnit;
  L.u_vscales = L.u_codes + kUnit * L.code_row;
  L.unit_bytes = L.u_vscales + kVScalesUnit;
  L.page_bytes = 2 * L.unit_bytes;
  *out = L;
  return TP_OK;
}

int validate_pool(const tp_page_pool* pool, Layout* L) {
  if (!pool) return fail(TP_ERR_INVALID, "page pool is NULL");
  int st = make_layout(pool->fmt, L);
  if (st != TP_OK) return st;
  if (pool->num_kv_heads <= 0) return fail(TP_ERR_INVALID, "num_kv_heads must be positive");
  if (pool->page_capacity < 0) return fail(TP_ERR_INVALID, "page_capacity must be >= 0");
  if (pool->page_capacity > 0) {
    if (!pool->pages) return fail(TP_ERR_INVALID, "page pool has NULL pages");
    if (reinterpret_cast<uintptr_t>(pool->pages) & 15) return fail(TP_ERR_INVALID, "page pool must be 16-byte aligned");
    if (pool->fmt.int8_radii && !pool->radii_scales) return fail(TP_ERR_INVALID, "int8 radii require radii_scales");
  }
  return TP_OK;
}

int validate_store(const tp_block_store* ref, Layout* L, bool keys) {
  if (!ref) return fail(TP_ERR_INVALID, "block store is NULL");
  int st = make_layout(ref->fmt, L);
  if (st != TP_OK) return st;
  if (ref->num_kv_heads <= 0) return fail(TP_ERR_INVALID, "num_kv_heads must be positive");
  if (ref->page_capacity < 0) return fail(TP_ERR_INVALID, "page_capacity must be >= 0");
  if (ref->page_capacity > 0) {
    if (!ref->v_codes || !ref->v_scales) return fail(TP_ERR_INVALID, "block store has a NULL value field");
    if (keys) {
      if (!ref->radii) return fail(TP_ERR_INVALID, "block store has NULL radii");
      if (L->l1_row > 0 && !ref->angle_codes_l1) return fail(TP_ERR_INVALID, "angle_codes_l1 is NULL");
      if (L->deep_row > 0 && !ref->angle_codes_deep) return fail(TP_ERR_INVALID, "angle_codes_deep is NULL");
      if (ref->fmt.int8_radii && !ref->radii_scales) return fail(TP_ERR_INVALID, "int8 radii require radii_scales");
    }
  }
  return TP_OK;
}

template <typename T>
__global__ void __launch_bounds__(256) encode_pages_kernel(PoolArgs P, const T* k, const T* v, int64_t head_stride,
                                                           int64_t token_stride, int64_t src_token0, int dst_page,
                                                           int n_pages, int32_t* d_state) {
  __shared__ uint8_t s_codes[kPage * kPairs];
  __shared__ float s_red[8];
  __shared__ __align__(16) uint8_t s_page[kMaxPageBytes];
  __shared__ __half s_rscale;
  const int p = blockIdx.x, h = blockIdx.y;
  const int64_t tok0 = src_token0 + int64_t(p) * kPage;
  encode_page<T>(k + h * head_stride + tok0 * token_stride, v + h * head_stride + tok0 * token_stride, token_stride,
                 P, s_page, &s_rscale, s_codes, s_red);
  store_page_block(P, s_page, s_rscale, h, dst_page + p);
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
  __shared__ __align__(16) uint8_t s_page[kMaxPageBytes];
  __shared__ __half s_rscale;
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
    encode_page<T>(tk, tv, kD, P, s_page, &s_rscale, s_codes, s_red);
    store_page_block(P, s_page, s_rscale, h, n_pages);
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

int tp_version(void) { return 3; }

int tp_row_bytes(const tp_format* fmt, int32_t* l1_row_bytes, int32_t* deep_row_bytes) {
  if (!fmt) return fail(TP_ERR_INVALID, "format is NULL");
  Layout L;
  int st = make_layout(*fmt, &L);
  if (st != TP_OK) return st;
  if (l1_row_bytes) *l1_row_bytes = L.l1_row;
  if (deep_row_bytes) *deep_row_bytes = L.deep_row;
  return TP_OK;
}

int tp_unit_bytes(const tp_format* fmt, int32_t* unit_bytes) {
  if (!fmt) return fail(TP_ERR_INVALID, "format is NULL");
  Layout L;
  int st = make_layout(*fmt, &L);
  if (st != TP_OK) return st;
  if (unit_bytes) *unit_bytes = L.unit_bytes;
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
