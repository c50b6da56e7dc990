// Shared device/host helpers of libturbopolar (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/turbopolar.h"

namespace tp {

// ----------------------------------------------------------------------------- errors
void set_error(const std::string& msg);
int fail(int status, const std::string& msg);
int check_launch(const char* what);

// ----------------------------------------------------------------------------- format
constexpr int kPage = TP_PAGE_TOKENS;  // tokens per page
constexpr int kD = TP_HEAD_DIM;        // head dim
constexpr int kPairs = kD / 2;
constexpr int kUnit = kPage / 2;       // tokens per unit (half page)
constexpr int64_t kVCodesPage = kPage * kD;   // int8 bytes per page per head
constexpr int64_t kVScalesPage = kPage * 4 * 2;  // fp16 [64][4]
constexpr int kVCodesUnit = kUnit * kD;       // 4096
constexpr int kVScalesUnit = kUnit * 4 * 2;   // 256

struct Layout {
  int l1_pairs, deep_pairs;      // pairs coded at level 1 / deep
  int l1_row, deep_row;          // packed bytes per token row
  int code_row;                  // l1_row + deep_row: one token's codes in a unit
  int radii_row;                 // bytes per token row of radii (128 fp16, 64 int8)
  int u_vcodes, u_codes, u_vscales, unit_bytes;  // byte offsets inside a unit, unit size
  int page_bytes;                // 2 * unit_bytes
};
// Returns TP_OK or TP_ERR_UNSUPPORTED.
int make_layout(const tp_format& f, Layout* out);
// Checks a pool's format, sizes and pointers.
int validate_pool(const tp_page_pool* pool, Layout* L);
// Checks a reference-layout block store (key fields only when `keys`).
int validate_store(const tp_block_store* ref, Layout* L, bool keys);

// Device view of a page pool.
struct PoolArgs {
  uint8_t* pages;
  __half* radii_scales;
  int num_kv_heads, page_capacity;
  int l1_bits, deep_bits, split_dim, int8_radii;
  int l1_pairs, l1_row, deep_row, code_row, radii_row;
  int u_vcodes, u_codes, u_vscales, unit_bytes, page_bytes;

  __host__ __device__ uint8_t* page(int h, int p) const {
    return pages + (int64_t(h) * page_capacity + p) * page_bytes;
  }
  __host__ __device__ __half* radii_scale(int h, int p) const {
    return int8_radii ? radii_scales + int64_t(h) * page_capacity + p : nullptr;
  }
};

inline PoolArgs pool_args(const tp_page_pool& p, const Layout& L) {
  PoolArgs a;
  a.pages = static_cast<uint8_t*>(p.pages);
  a.radii_scales = static_cast<__half*>(p.radii_scales);
  a.num_kv_heads = p.num_kv_heads;
  a.page_capacity = p.page_capacity;
  a.l1_bits = p.fmt.l1_bits;
  a.deep_bits = p.fmt.deep_bits;
  a.split_dim = p.fmt.split_dim;
  a.int8_radii = p.fmt.int8_radii;
  a.l1_pairs = L.l1_pairs;
  a.l1_row = L.l1_row;
  a.deep_row = L.deep_row;
  a.code_row = L.code_row;
  a.radii_row = L.radii_row;
  a.u_vcodes = L.u_vcodes;
  a.u_codes = L.u_codes;
  a.u_vscales = L.u_vscales;
  a.unit_bytes = L.unit_bytes;
  a.page_bytes = L.page_bytes;
  return a;
}

// ----------------------------------------------------------------------------- page layout in HBM
// The codes are the reference's, bit for bit; their placement is chosen for the decode kernel
// (tp_export_pages / tp_import_pages convert to and from the reference layout).  A page block
// is two units (tokens 0-31, 32-63) of PoolArgs::unit_bytes each; inside a unit, for token
// row l = 0..31:
//
// * radii at offset 0: float16 rows of 128 bytes, 16-byte chunk c (pairs 8c..8c+7) stored at
//   chunk c ^ (l & 7), the XOR swizzle that makes the kernel's row-fragment loads bank-conflict
//   free once a unit is copied linearly into shared memory; int8 radii rows are 64 bytes, linear.
// * value codes at u_vcodes, stored as (code ^ 0x80) -- i.e. code + 128 as a byte -- in mma
//   fragment order: token l = 16*kk + 8*a + 2*t + b (kk: 16-token step, a: upper/lower 8,
//   t: lane quad column, b: pair bit) and channel d = 32*G + 4*g + 2*e_hi + e_lo sit at byte
//   kk*2048 + G*512 + g*64 + t*16 + a*8 + e_hi*4 + e_lo*2 + b, so lane 4g+t of a warp finds its
//   whole A fragment for group G of step kk in one 16-byte word.
// * angle codes at u_codes: code_row bytes per token, level-1 codes then deep codes, each
//   packed as the reference packs them (4-bit: even index in the low nibble; 2-bit: LSB first).
// * value scales at u_vscales (float16, one per token and 32-channel group) at half index
//   kk*64 + t*16 + a*8 + G*2 + b, so a lane reads (scale[tok][G], scale[tok+1][G]) pairs for its
//   two token pairs with two 16-byte loads.
__host__ __device__ __forceinline__ int radii_f16_offset(int l, int j) {  // bytes, l < 32
  return l * 128 + ((((j >> 3) ^ (l & 7))) << 4) + (j & 7) * 2;
}
__host__ __device__ __forceinline__ int vcode_offset(int l, int d) {  // bytes, l < 32
  const int kk = l >> 4, r = l & 15, a = r >> 3, t = (r >> 1) & 3, b = r & 1;
  const int G = d >> 5, g = (d >> 2) & 7, e_hi = (d >> 1) & 1, e_lo = d & 1;
  return kk * 2048 + G * 512 + g * 64 + t * 16 + a * 8 + e_hi * 4 + e_lo * 2 + b;
}
__host__ __device__ __forceinline__ int vscale_index(int l, int G) {  // halves, l < 32
  const int kk = l >> 4, r = l & 15, a = r >> 3, t = (r >> 1) & 3, b = r & 1;
  return kk * 64 + t * 16 + a * 8 + G * 2 + b;
}

// Addresses of token l (0..63) of a page block `pg` (global or shared memory).
template <class LAY>
__host__ __device__ __forceinline__ uint8_t* unit_of(const LAY& L, uint8_t* pg, int l) {
  return pg + (l >> 5) * L.unit_bytes;
}
template <class LAY>
__host__ __device__ __forceinline__ __half* radius_f16_at(const LAY& L, uint8_t* pg, int l, int j) {
  return reinterpret_cast<__half*>(unit_of(L, pg, l) + radii_f16_offset(l & 31, j));
}
template <class LAY>
__host__ __device__ __forceinline__ int8_t* radius_i8_at(const LAY& L, uint8_t* pg, int l, int j) {
  return reinterpret_cast<int8_t*>(unit_of(L, pg, l) + (l & 31) * kPairs + j);
}
template <class LAY>
__host__ __device__ __forceinline__ uint8_t* codes_at(const LAY& L, uint8_t* pg, int l) {  // level-1 then deep
  return unit_of(L, pg, l) + L.u_codes + (l & 31) * L.code_row;
}
template <class LAY>
__host__ __device__ __forceinline__ uint8_t* vcode_at(const LAY& L, uint8_t* pg, int l, int d) {
  return unit_of(L, pg, l) + L.u_vcodes + vcode_offset(l & 31, d);
}
template <class LAY>
__host__ __device__ __forceinline__ __half* vscale_at(const LAY& L, uint8_t* pg, int l, int G) {
  return reinterpret_cast<__half*>(unit_of(L, pg, l) + L.u_vscales) + vscale_index(l & 31, G);
}

// ----------------------------------------------------------------------------- device helpers
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Pack two floats to a half2 register (lo = a, hi = b), round to nearest.
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(b), "f"(a));
  return d;
}

// D = A(16x16, row) * B(16x8, col) + C, fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Transpose an 8x8 b16 matrix held one row-pair per lane (row lane/4, cols 2*(lane%4)+{0,1}).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// ----------------------------------------------------------------------------- bulk copies
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Invalidate a barrier with no pending arrivals or transactions, before initialising it again.
__device__ __forceinline__ void mbar_inval(uint64_t* bar) {
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
// Make barrier initialisation visible to the async proxy (bulk copies complete on it).
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
// Order this thread's earlier generic-proxy shared-memory accesses before later async-proxy ones.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
// One bounded-time probe of phase `parity`; true once that phase has completed.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// 1-D bulk copy global -> this CTA's shared memory completing on `bar`.  16-byte aligned, size % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// L2 policy for data read exactly once per launch: evicted first, so streaming pages do not
// push the kernels' code, counters and partial records out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}
// bulk_g2s with an L2 cache policy.
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;\n" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// Tiled 3-D tensor copy global -> this CTA's shared memory (TMA) of the box at element coordinates
// (x, y, z) of the tensor map at generic address `tmap`, completing on `bar`.  x times the
// element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar,
                                            uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Correctly rounded float32 value of a float64 expression, as the codec's transcendental model.
__device__ __forceinline__ float d2f(double x) { return __double2float_rn(x); }

}  // namespace tp
