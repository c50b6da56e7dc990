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
struct Layout {
  int l1_pairs, deep_pairs;      // pairs coded at level 1 / deep
  int l1_row, deep_row;          // packed bytes per token row
  int radii_row;                 // bytes per token row of radii (128 fp16, 64 int8)
  int64_t radii_page, l1_page, deep_page;  // bytes per page per head
};
// Returns TP_OK or TP_ERR_UNSUPPORTED.
int make_layout(const tp_format& f, Layout* out);
// Checks a pool's format, sizes and pointers (key fields only when `keys`).
int validate_pool(const tp_page_pool* pool, Layout* L, bool keys = true);

constexpr int kPage = TP_PAGE_TOKENS;  // tokens per page
constexpr int kD = TP_HEAD_DIM;        // head dim
constexpr int kPairs = kD / 2;
constexpr int64_t kVCodesPage = kPage * kD;   // int8 bytes per page per head
constexpr int64_t kVScalesPage = kPage * 4 * 2;  // fp16 [64][4]

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

__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Correctly rounded float32 value of a float64 expression, as the codec's transcendental model.
__device__ __forceinline__ float d2f(double x) { return __double2float_rn(x); }

}  // namespace tp
