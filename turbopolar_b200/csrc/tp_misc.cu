// Secondary kernels: scores-only attention and page decompression.
#include "tp_codec.cuh"

namespace tp {


// A reference-layout block store (tp_block_store) on the device.
struct RefView {
  uint8_t* radii;
  __half* radii_scales;
  uint8_t* l1;
  uint8_t* deep;
  int8_t* v_codes;
  __half* v_scales;
  int page_capacity;
};

static RefView ref_view(const tp_block_store& r) {
  RefView v;
  v.radii = static_cast<uint8_t*>(r.radii);
  v.radii_scales = static_cast<__half*>(r.radii_scales);
  v.l1 = static_cast<uint8_t*>(r.angle_codes_l1);
  v.deep = static_cast<uint8_t*>(r.angle_codes_deep);
  v.v_codes = static_cast<int8_t*>(r.v_codes);
  v.v_scales = static_cast<__half*>(r.v_scales);
  v.page_capacity = r.page_capacity;
  return v;
}

// float32 (cos, sin) of every code of both code sets; the decoder's angle formula in float32
// (rfsn_v11/quant/polar/decoder.py:36-56).
__device__ void build_cos_sin(float2* tab, int l1_bits, int deep_bits) {
  for (int i = threadIdx.x; i < 512; i += blockDim.x) {
    const int bits = i < 256 ? l1_bits : deep_bits;
    const int code = i & 255;
    tab[i] = code < (1 << bits) ? cos_sin_of_code(code, bits) : make_float2(0.f, 0.f);
  }
}

// Decoded float16 key pair j of token l of page block pg: fp16(r * cos), fp16(r * sin) with the
// float32 products of decoder.py:57-67.
__device__ __forceinline__ __half2 decode_pair(const PoolArgs& V, const float2* tab, uint8_t* pg, __half rscale, int l,
                                               int j) {
  uint32_t code;
  const float2* t;
  const uint8_t* row = codes_at(V, pg, l);
  if (j < V.l1_pairs) {
    code = V.l1_bits == 8 ? row[j] : (row[j >> 1] >> (4 * (j & 1))) & 15u;
    t = tab;
  } else {
    const int rel = j - V.l1_pairs;
    row += V.l1_row;
    if (V.deep_bits == 8) code = row[rel];
    else if (V.deep_bits == 4) code = (row[rel >> 1] >> (4 * (rel & 1))) & 15u;
    else code = (row[rel >> 2] >> (2 * (rel & 3))) & 3u;
    t = tab + 256;
  }
  float r;
  if (V.int8_radii) {
    const float arg = __fmul_rn(float(*radius_i8_at(V, pg, l, j)), __half2float(rscale));
    r = d2f(exp(double(arg)));
  } else {
    r = __half2float(*radius_f16_at(V, pg, l, j));
  }
  const float2 cs = t[code];
  return __halves2half2(__float2half_rn(__fmul_rn(r, cs.x)), __float2half_rn(__fmul_rn(r, cs.y)));
}

// One CTA per (page, KV head); thread l = token.  Scores accumulate in float32 over the
// float16-rounded decoded key.
__global__ void fused_scores_kernel(PoolArgs V, const void* q, int q_f32, int num_q_heads, int group, float scale,
                                    int n_pages, __half* scores) {
  __shared__ float2 tab[512];
  __shared__ float qs[8][kD];
  build_cos_sin(tab, V.l1_bits, V.deep_bits);
  const int p = blockIdx.x, h = blockIdx.y, l = threadIdx.x;
  uint8_t* pg = V.page(h, p);
  const __half rscale = V.int8_radii ? *V.radii_scale(h, p) : __half(0.f);
  for (int g0 = 0; g0 < group; g0 += 8) {
    const int gc = min(8, group - g0);
    __syncthreads();
    for (int i = threadIdx.x; i < gc * kD; i += blockDim.x) {
      const int64_t idx = int64_t(h * group + g0 + i / kD) * kD + i % kD;
      qs[i / kD][i % kD] = q_f32 ? __half2float(__float2half_rn(static_cast<const float*>(q)[idx]))
                                 : __half2float(static_cast<const __half*>(q)[idx]);
    }
    __syncthreads();
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < kPairs; ++j) {
      const float2 k = __half22float2(decode_pair(V, tab, pg, rscale, l, j));
#pragma unroll
      for (int hh = 0; hh < 8; ++hh)
        if (hh < gc) acc[hh] = fmaf(qs[hh][2 * j], k.x, fmaf(qs[hh][2 * j + 1], k.y, acc[hh]));
    }
    for (int hh = 0; hh < gc; ++hh)
      scores[int64_t(h * group + g0 + hh) * n_pages * kPage + int64_t(p) * kPage + l] = __float2half_rn(acc[hh] * scale);
  }
}

// One CTA per (page, KV head), 256 threads: thread (token l, quarter c) writes key pairs
// [16c, 16c+16) and values [32c, 32c+32) of token l.
__global__ void decode_pages_kernel(PoolArgs V, int first_page, int n_pages, __half* k_out, __half* v_out) {
  __shared__ float2 tab[512];
  build_cos_sin(tab, V.l1_bits, V.deep_bits);
  __syncthreads();
  const int p = blockIdx.x, h = blockIdx.y;
  const int l = threadIdx.x >> 2, c = threadIdx.x & 3;
  uint8_t* pg = V.page(h, first_page + p);
  const int64_t orow = (int64_t(h) * n_pages + p) * kPage + l;
  if (k_out) {
    const __half rscale = V.int8_radii ? *V.radii_scale(h, first_page + p) : __half(0.f);
    __half2* ko = reinterpret_cast<__half2*>(k_out + orow * kD);
    for (int i = 0; i < 16; ++i) ko[16 * c + i] = decode_pair(V, tab, pg, rscale, l, 16 * c + i);
  }
  const float s = __half2float(*vscale_at(V, pg, l, c));
  __half* vo = v_out + orow * kD + 32 * c;
  for (int i = 0; i < 32; ++i) {
    const int8_t code = int8_t(*vcode_at(V, pg, l, 32 * c + i) ^ 0x80u);
    vo[i] = __float2half_rn(__fmul_rn(float(code), s));
  }
}

// Convert pages between the pool layout and the reference's block-storage layout
// (rfsn_v11/generation/storage.py:89-102, :160-169): radii rows unswizzled, level-1 and deep
// codes in their own arrays, value codes as plain int8 [token][channel], value scales
// [token][group].  One CTA per (page, head); thread (token l, quarter c).  to_ref: pool -> ref;
// otherwise ref -> pool.
__global__ void convert_pages_kernel(PoolArgs pool, RefView ref, int first_page, bool to_ref, bool keys) {
  const int p = blockIdx.x, h = blockIdx.y;
  const int l = threadIdx.x >> 2, c = threadIdx.x & 3;
  uint8_t* pg = pool.page(h, first_page + p);
  const int64_t rs = int64_t(h) * ref.page_capacity + p;
  if (keys) {
    if (pool.int8_radii) {
      int8_t* pr = radius_i8_at(pool, pg, l, 16 * c);
      int8_t* rr = reinterpret_cast<int8_t*>(ref.radii) + rs * kPage * 64 + l * 64 + 16 * c;
      for (int i = 0; i < 16; ++i) {
        if (to_ref) rr[i] = pr[i]; else pr[i] = rr[i];
      }
      if (threadIdx.x == 0) {
        __half* prs = pool.radii_scale(h, first_page + p);
        if (to_ref) ref.radii_scales[rs] = *prs; else *prs = ref.radii_scales[rs];
      }
    } else {
      for (int i = 0; i < 16; ++i) {
        const int j = 16 * c + i;
        __half* a = radius_f16_at(pool, pg, l, j);
        __half* b = reinterpret_cast<__half*>(ref.radii + rs * kPage * 128) + l * kPairs + j;
        if (to_ref) *b = *a; else *a = *b;
      }
    }
    uint8_t* row = codes_at(pool, pg, l);
    for (int i = c; i < pool.l1_row; i += 4) {
      uint8_t* r = ref.l1 + (rs * kPage + l) * pool.l1_row + i;
      if (to_ref) *r = row[i]; else row[i] = *r;
    }
    for (int i = c; i < pool.deep_row; i += 4) {
      uint8_t* r = ref.deep + (rs * kPage + l) * pool.deep_row + i;
      if (to_ref) *r = row[pool.l1_row + i]; else row[pool.l1_row + i] = *r;
    }
  }
  uint8_t* rv = reinterpret_cast<uint8_t*>(ref.v_codes) + rs * kVCodesPage;
  for (int i = 0; i < 32; ++i) {
    const int d = 32 * c + i;
    uint8_t* pv = vcode_at(pool, pg, l, d);
    if (to_ref) rv[l * kD + d] = *pv ^ 0x80u;
    else *pv = rv[l * kD + d] ^ 0x80u;
  }
  __half* rsc = ref.v_scales + rs * kPage * 4;
  __half* psc = vscale_at(pool, pg, l, c);
  if (to_ref) rsc[l * 4 + c] = *psc;
  else *psc = rsc[l * 4 + c];
}

}  // namespace tp

using namespace tp;

extern "C" {

int tp_fused_scores(const tp_page_pool* pool, int32_t n_pages, const void* q, int32_t q_dtype, int32_t num_q_heads,
                    float scale, void* scores, void* stream) {
  Layout L;
  int st = validate_pool(pool, &L);
  if (st != TP_OK) return st;
  if (num_q_heads <= 0 || num_q_heads % pool->num_kv_heads)
    return fail(TP_ERR_INVALID, "num_q_heads must be divisible by num_kv_heads for GQA");
  if (n_pages < 0 || n_pages > pool->page_capacity) return fail(TP_ERR_INVALID, "n_pages outside the page pool");
  if (!q || !scores) return fail(TP_ERR_INVALID, "tp_fused_scores: NULL argument");
  if (q_dtype != TP_F16 && q_dtype != TP_F32) return fail(TP_ERR_INVALID, "q must be float16 or float32");
  if (n_pages == 0) return TP_OK;
  dim3 grid(n_pages, pool->num_kv_heads);
  fused_scores_kernel<<<grid, kPage, 0, static_cast<cudaStream_t>(stream)>>>(
      pool_args(*pool, L), q, q_dtype == TP_F32, num_q_heads, num_q_heads / pool->num_kv_heads, scale, n_pages,
      static_cast<__half*>(scores));
  return check_launch("tp_fused_scores");
}

int tp_decode_pages(const tp_page_pool* pool, int32_t first_page, int32_t n_pages, void* k_out, void* v_out,
                    void* stream) {
  Layout L;
  int st = validate_pool(pool, &L);
  if (st != TP_OK) return st;
  if (first_page < 0 || n_pages < 0 || int64_t(first_page) + n_pages > pool->page_capacity)
    return fail(TP_ERR_INVALID, "tp_decode_pages: page range outside the pool");
  if (!v_out) return fail(TP_ERR_INVALID, "tp_decode_pages: NULL value output");
  if (n_pages == 0) return TP_OK;
  dim3 grid(n_pages, pool->num_kv_heads);
  decode_pages_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(pool_args(*pool, L), first_page, n_pages,
                                                                           static_cast<__half*>(k_out),
                                                                           static_cast<__half*>(v_out));
  return check_launch("tp_decode_pages");
}

static int convert(const tp_page_pool* pool, int32_t first_page, int32_t n_pages, const tp_block_store* ref,
                   bool to_ref, void* stream) {
  Layout L, LR;
  const bool keys = ref && ref->radii;
  int st = validate_pool(pool, &L);
  if (st != TP_OK) return st;
  st = validate_store(ref, &LR, keys);
  if (st != TP_OK) return st;
  if (pool->num_kv_heads != ref->num_kv_heads || pool->fmt.l1_bits != ref->fmt.l1_bits ||
      pool->fmt.deep_bits != ref->fmt.deep_bits || pool->fmt.split_dim != ref->fmt.split_dim ||
      pool->fmt.int8_radii != ref->fmt.int8_radii)
    return fail(TP_ERR_INVALID, "page conversion: pool and block store differ in heads or format");
  if (first_page < 0 || n_pages < 0 || int64_t(first_page) + n_pages > pool->page_capacity || n_pages > ref->page_capacity)
    return fail(TP_ERR_INVALID, "page conversion: page range outside a pool");
  if (n_pages == 0) return TP_OK;
  dim3 grid(n_pages, pool->num_kv_heads);
  convert_pages_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(pool_args(*pool, L), ref_view(*ref),
                                                                            first_page, to_ref, keys);
  return check_launch(to_ref ? "tp_export_pages" : "tp_import_pages");
}

int tp_export_pages(const tp_page_pool* pool, int32_t first_page, int32_t n_pages, const tp_block_store* ref,
                    void* stream) {
  return convert(pool, first_page, n_pages, ref, true, stream);
}

int tp_import_pages(const tp_page_pool* pool, int32_t first_page, int32_t n_pages, const tp_block_store* ref,
                    void* stream) {
  return convert(pool, first_page, n_pages, ref, false, stream);
}

}  // extern "C"
