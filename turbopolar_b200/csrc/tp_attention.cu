// Fused decode attention over compressed KV pages + dense tail (sm_100a).
//
// Replaces the reference's Metal kernels tqpolar_online_attention_quant_v[_dense_tail]
// (rfsn_v11/kernels/turbo_polar/tqpolar_online_attention.metal:197-629) with the numerics of
// the bridge's CPU fallback (rfsn_v11/kernels/turbo_polar/metal.py:293-332) as the target.
//
// Work decomposition.  A "unit" is one half page (32 tokens) of one (KV head, query chunk of
// at most 8 heads): one contiguous block of the page pool.  The units of all heads form one flat
// list cut into gridDim.x contiguous ranges, one per CTA (one CTA per SM), so every SM streams
// the same number of bytes whatever the head count or context length; a range spans at most
// two heads ("segments").  Inside a CTA, 7 compute warps take units w, w+7, ... of the range
// and one copy warp streams them: lane w issues one cp.async.bulk per unit of compute warp w
// into that warp's own ring stages (full/empty mbarriers per stage), so no wait ever runs
// ahead of its barrier's phase and compute warps never wait on one another.
//
// Per half page a compute warp computes, with mma.sync m16n8k16 (fp16 in, fp32 accumulate):
//   S^T[token][head] = K[token][dim] . Q^T[dim][head]      M = 16 tokens, N = 8 query heads
// where every lane decodes exactly the key pairs its A fragment holds: lane (g, t) owns pairs
// [16t, 16t+16) of tokens g and g+8, each pair k = radius * (cos, sin)(code) from a 16-entry
// half2 table, so no decoded key ever touches shared memory.  Online softmax runs in the
// base-2 domain on the accumulator fragments; P is converted to fp16 and transposed into the
// B operand with movmatrix, the per-(token, 32-channel group) value scales are folded into
// P (one copy of B per group), and
//   O^T[dim][head] += V'^T[dim][token] . (P * scale_g)^T[token][head]
// runs with V' = code + 1152 produced by a byte permute into the fp16 exponent (0x64xx = 1024
// + byte, byte = code ^ 0x80).  The bias is removed at the end with a ones-row tile per group
// that accumulates sum_t P*scale_g alongside (O = O' - 1152 * sum).
//
// Split combine.  The warps of a CTA merge through shared memory and the CTA writes one
// partial (m, l, o[128]) per query head and segment to the workspace.  A second kernel, launched
// as a programmatic dependent of the page pass, computes the dense-tail partial (and, in a
// decode step, appends the new token) while the page pass runs, then waits for it to complete
// and merges the partials of each query head into the fp16 output (sharded: with the other
// ranks' records, exchanged over NVLink in the same launch).
//
// Dense-V variant (tp_decode_attention_dense_v; the reference's tqpolar_online_attention_dense_v,
// tqpolar_online_attention.metal:10-195): compressed keys, float16 values in a separate
// [head][token][128] array.  A stage holds the unit's radii and angle codes (two bulk copies)
// and its 32 value rows (two TMA tensor copies of 32 tokens x 64 channels, 128-byte swizzle), and
// P.V multiplies the value rows as they are, with P as float16 hi + lo parts.
#include <cfloat>
#include <cstring>
#include <cmath>
#include <functional>
#include <mutex>
#include <thread>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "tp_codec.cuh"
#include "tp_overlap.h"

namespace tp {

#ifndef TP_CONSUMERS
#define TP_CONSUMERS 7
#endif
#ifndef TP_COPY_SPLIT
#define TP_COPY_SPLIT 1
#endif
// TP_QK_CUDA_CORES=1 builds the comparison variant of the default-format page pass whose Q.K
// product runs on CUDA cores (float32 FMA over the same decoded key fragments, quad shuffles;
// P.V unchanged; at most 4 query heads per KV head) instead of mma.sync.  Off in the product.
#ifndef TP_QK_CUDA_CORES
#define TP_QK_CUDA_CORES 0
#endif
// Key formats whose page pass computes P.V exactly (bit kMode set; see process_half): the
// values dequantised as the reference rounds them, fp16(code * scale), and the softmax weights
// as float16 hi + lo parts.  The others fold the value scale into float16 weights.
#ifndef TP_EXACT_PV
#define TP_EXACT_PV 4
#endif
constexpr int kConsumers = TP_CONSUMERS;             // page-pass compute warps
constexpr int kCopySplit = TP_COPY_SPLIT;            // copy-warp lanes (and bulk copies) per unit
constexpr int kIssuers = kConsumers * kCopySplit;    // issuing lanes of the copy warp(s)
constexpr int kProducerWarps = (kIssuers + 31) / 32;
constexpr int kThreads = (kConsumers + kProducerWarps) * 32;
constexpr int kMaxStages = 24;                   // ring stages (one unit each)
constexpr int kMaxHeads = 8;  // query heads per unit (N of the mma)
constexpr int kHalf = 32;     // tokens per unit
// Records exchanged between CTAs and between GPUs: (m, l, o[128]) per query head, padded to
// 132 floats so each starts on 16 bytes (staged with 16-byte copies).
constexpr int kRecFloats = 132;
constexpr int kPartialStride = kMaxHeads * kRecFloats;  // floats per workspace slot
constexpr int kLutEntries = 256;
constexpr int kMaxContrib = 192;  // CTAs that can share one (KV head, query chunk) segment

struct AttnParams {
  const uint8_t* pages;
  const __half* radii_scales;
  int page_capacity;
  int l1_bits, deep_bits, l1_pairs, l1_row, deep_row, code_row, radii_row, int8_radii;
  int unit_bytes;  // bytes per half page (one bulk copy)
  void* tail_k;
  void* tail_v;
  int tail_f32;
  tp_state st;
  int32_t* d_state;  // written only by the fused step
  const void* q;
  int q_f32;
  int num_q_heads, num_kv_heads, group, nqc, gmax;
  int main_grid;  // CTAs of the page pass
  // Whole-segment partition (more (KV head, query chunk) segments than CTAs): CTA c streams
  // whole segments and writes one merged record per segment, at workspace slot = segment.
  int owner;
  // The previous call launched on this stream writes nothing this call reads: the page pass
  // streams before griddepcontrol.wait (the host decides: StreamLog in tp_overlap.h).
  int spec;
  // With spec: no call that may still be running uses this call's workspace, so the page pass
  // writes its partials first and waits for the previous kernel only before it exits.
  int ws_private;
  // No call that may still be running writes this call's state words, pages or radius scales:
  // what the page pass reads of them before griddepcontrol.wait is final (StreamLog's probe).
  int cache_final;
  // Fused decode step: one new token per KV head (k_new/v_new, tail dtype, heads
  // new_head_stride elements apart) appended before attention; wpool is the writable pool.
  int fused;
  const void* k_new;
  const void* v_new;
  int64_t new_head_stride;
  PoolArgs wpool;
  // Cross-GPU exchange (sequence sharding): xworld ranks; xbuf[r] is rank r's exchange buffer
  // mapped into this process; xworld == 0 without an exchange.
  int xworld, xrank;
  uint8_t* xbuf[TP_MAX_RANKS];
  float scale_log2;
  __half* out;
  float* partial_out;
  float* ws_partials;
  int* ws_error;
  int stage_bytes, off_vcodes, off_codes, off_vscales;  // a stage holds one unit as laid out in the pool
  int smem_bar_off, smem_lut_off, smem_merge_off, smem_stage_off;
  int smem_scale_off;  // float radius scale of the unit in each ring stage (int8 radii)
  int smem_tab_off;    // adapter format: the deep (cos, sin) table, 16 copies
  int smem_qcc_off;    // TP_QK_CUDA_CORES: float32 query heads per compute warp
  int n_stages;  // ring stages of the page pass
  int lut_deep;  // shared-memory float2 (cos, sin) tables: level-1 entries, then deep from here
  // Decoder tables computed on the host (code / (2^bits - 1) * 2pi - pi in float32, cos and sin
  // rounded to float32; decoder.py:36-56): the fast path's 16 entries as float16 hi / lo parts
  // (uint2 (cos_hi, sin_hi), (cos_lo, sin_lo)) in the first 16 slots, or the adapter path's 256
  // deep entries as float2.  The general path builds its tables on the device.
  float2 cs[kLutEntries];
  // Dense-V variant: a stage holds the unit's radii at 0 (k_radii_bytes), its angle codes at
  // off_codes (k_code_bytes, copied from unit offset k_src_codes) and its value rows at
  // off_vdense (1024-byte aligned: two 4 KB boxes, channels 0-63 then 64-127, each token row
  // 128 bytes with 16-byte chunk c stored at c ^ (row & 7)); vmap is the tensor map of the value
  // array {128 channels, tokens, KV heads}.
  int k_radii_bytes, k_code_bytes, k_src_codes, off_vdense;
  CUtensorMap vmap;
};

// Work partition: the U units (half pages, head-major, uph per head) are cut into C = min(U,
// grid) ranges; CTA cc owns [floor(cc*U/C), floor((cc+1)*U/C)).  With U = k*C + r,
// floor(cc*U/C) = cc*k + floor(cc*r/C) and cc*r < C^2 fits in 32 bits, so the device does
// neither 64-bit nor floating-point division (both are long or slow instruction sequences).
struct Grid {
  int uph, U, C, k, r;
};

__device__ __forceinline__ Grid grid_of(int num_vh, int n_pages, int grid) {
  Grid g;
  g.uph = 2 * n_pages;
  g.U = num_vh * g.uph;
  g.C = g.U < grid ? g.U : grid;
  g.k = g.C > 0 ? g.U / g.C : 0;
  g.r = g.C > 0 ? g.U - g.k * g.C : 0;
  return g;
}

__device__ __forceinline__ int part_begin(const Grid& g, int cc) { return cc * g.k + (cc * g.r) / g.C; }

// The CTA whose range holds unit u (0 <= u < U): a float estimate, exact within one, then
// corrected against part_begin.
__device__ __forceinline__ int part_owner(const Grid& g, int u) {
  int c = int(float(u) * float(g.C) / float(g.U));
  c = min(max(c, 0), g.C - 1);
  while (c + 1 < g.C && part_begin(g, c + 1) <= u) ++c;
  while (c > 0 && part_begin(g, c) > u) --c;
  return c;
}

__device__ __forceinline__ int64_t clamp64(int64_t x, int64_t lo, int64_t hi) { return x < lo ? lo : (x > hi ? hi : x); }

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint2 lds64(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
  return h2_as_u32(__hmul2(u32_as_h2(a), u32_as_h2(b)));
}

// Byte offset of 16-byte chunk `c` of row `r` in a swizzled 128-byte-row tile.
__device__ __forceinline__ int swz128(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// ----------------------------------------------------------------------------- per-warp state
struct WarpAcc {
  float o[8][4];     // O'^T tiles: tile md rows d = 32(md/2) + 4g + 2(md%2) (+1), cols heads 2t, 2t+1
  float ones[4][4];  // per value group: sum_t P*scale (every row identical)
  float m[2], l[2];  // running max (log2 units) and lane-partial sum for heads 2t, 2t+1
};

__device__ __forceinline__ void acc_reset(WarpAcc& A) {
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) A.o[i][j] = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) A.ones[i][j] = 0.f;
  A.m[0] = A.m[1] = -INFINITY;
  A.l[0] = A.l[1] = 0.f;
}

// Online-softmax update from the raw score fragments of NT 16-token tiles; returns P in sc.
template <int NT, bool kOnes>
__device__ __forceinline__ void softmax_update(WarpAcc& A, float (&sc)[NT][4], float c) {
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int mt = 0; mt < NT; ++mt) {
    mx0 = fmaxf(mx0, fmaxf(sc[mt][0], sc[mt][2]));
    mx1 = fmaxf(mx1, fmaxf(sc[mt][1], sc[mt][3]));
  }
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
  }
  const float mn0 = fmaxf(A.m[0], mx0 * c), mn1 = fmaxf(A.m[1], mx1 * c);
  const float b0 = (mn0 == -INFINITY) ? 0.f : mn0, b1 = (mn1 == -INFINITY) ? 0.f : mn1;
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int mt = 0; mt < NT; ++mt) {
    sc[mt][0] = exp2_approx(fmaf(sc[mt][0], c, -b0));
    sc[mt][1] = exp2_approx(fmaf(sc[mt][1], c, -b1));
    sc[mt][2] = exp2_approx(fmaf(sc[mt][2], c, -b0));
    sc[mt][3] = exp2_approx(fmaf(sc[mt][3], c, -b1));
    s0 += sc[mt][0] + sc[mt][2];
    s1 += sc[mt][1] + sc[mt][3];
  }
  if (mn0 != A.m[0] || mn1 != A.m[1]) {
    const float al0 = exp2_approx(A.m[0] - b0), al1 = exp2_approx(A.m[1] - b1);
    A.l[0] *= al0;
    A.l[1] *= al1;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      A.o[i][0] *= al0; A.o[i][2] *= al0;
      A.o[i][1] *= al1; A.o[i][3] *= al1;
    }
    if (kOnes) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        A.ones[i][0] *= al0; A.ones[i][2] *= al0;
        A.ones[i][1] *= al1; A.ones[i][3] *= al1;
      }
    }
    A.m[0] = mn0;
    A.m[1] = mn1;
  }
  A.l[0] += s0;
  A.l[1] += s1;
}

// ----------------------------------------------------------------------------- key decode
// Every path decodes a key pair as the reference decoder does (decoder.py:57-67): the float32
// radius times the float32 (cos, sin) of the code angle, each product rounded once to float16,
// so the keys the kernel multiplies are the reference's decoded keys.
//
// Fast path: default format (level-1 and deep both 4-bit, split_dim 64, float16 radii).  Entry
// c of the table at shared address tab_sa (256-byte aligned) holds the float32 cos and sin of
// code c split into float16 parts, (cos_hi, sin_hi) then (cos_lo, sin_lo), hi = fp16(v) and
// lo = fp16(v - hi).  A pair is fma(r, hi, r * lo) in half2: one rounding of r * (hi + lo), and
// hi + lo carries the float32 value to about 2^-22, so the key is fp16(r * cos) as the reference
// decodes it, except when r * cos lies within that distance of a float16 rounding boundary.
// Entry addresses: each code byte's nibbles are pre-scaled by 8 in place (two masks per four
// bytes), and one byte permute splices a scaled nibble into the table's address.  Writes the 16
// decoded pairs [16t, 16t+16) of stage row `r` as half2 (x, y).
__device__ __forceinline__ void decode_row_fast(const uint8_t* stage, const AttnParams& P, uint32_t tab_sa,
                                                int r, int t, uint32_t (&kp)[16]) {
  const uint4 R0 = lds128(stage + swz128(r, 2 * t));
  const uint4 R1 = lds128(stage + swz128(r, 2 * t + 1));
  const uint2 C = lds64(stage + P.off_codes + r * 32 + 8 * t);
  const uint32_t rw[8] = {R0.x, R0.y, R0.z, R0.w, R1.x, R1.y, R1.z, R1.w};
  const uint32_t lo[2] = {(C.x << 3) & 0x78787878u, (C.y << 3) & 0x78787878u};
  const uint32_t hi[2] = {(C.x >> 1) & 0x78787878u, (C.y >> 1) & 0x78787878u};
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int n = i & 7;
    const uint32_t src = (n & 1) ? hi[i >> 3] : lo[i >> 3];
    const uint32_t addr = prmt(src, tab_sa, 0x7650u | uint32_t(n >> 1));  // tab_sa + 8 * nibble
    uint2 e;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(e.x), "=r"(e.y) : "r"(addr));
    const __half2 rp = u32_as_h2(rw[i >> 1]);
    const __half2 rr = (i & 1) ? __high2half2(rp) : __low2half2(rp);
    kp[i] = h2_as_u32(__hfma2(rr, u32_as_h2(e.x), __hmul2(rr, u32_as_h2(e.y))));
  }
}

// General path: any supported format.  Tables: level-1 at cs[0..], deep at cs[P.lut_deep..].
__device__ __forceinline__ void decode_row_general(const uint8_t* stage, const AttnParams& P, const float2* cs,
                                                   float radius_scale, int r, int t, uint32_t (&kp)[16]) {
  const uint8_t* l1row = stage + P.off_codes + r * P.code_row;
  const uint8_t* deeprow = l1row + P.l1_row;
#pragma unroll 4
  for (int i = 0; i < 16; ++i) {
    const int j = 16 * t + i;
    uint32_t code;
    float2 c;
    if (j < P.l1_pairs) {
      if (P.l1_bits == 8) code = l1row[j];
      else code = (l1row[j >> 1] >> (4 * (j & 1))) & 15u;
      c = cs[code];
    } else {
      const int rel = j - P.l1_pairs;
      if (P.deep_bits == 8) code = deeprow[rel];
      else if (P.deep_bits == 4) code = (deeprow[rel >> 1] >> (4 * (rel & 1))) & 15u;
      else code = (deeprow[rel >> 2] >> (2 * (rel & 3))) & 3u;
      c = cs[P.lut_deep + code];
    }
    float rad;
    if (P.int8_radii) {
      const int8_t rc = reinterpret_cast<const int8_t*>(stage)[r * 64 + j];
      rad = __expf(float(rc) * radius_scale);
    } else {
      rad = __half2float(reinterpret_cast<const __half*>(stage + swz128(r, j >> 3))[j & 7]);
    }
    kp[i] = pack_h2(rad * c.x, rad * c.y);
  }
}

// Adapter path: log-int8 radii, split_dim 0 and 8-bit angle codes (the format the Llama
// adapter uses, benchmarks/turbopolar_fast_attention.py:217-228).  Radius of int8 code c:
// exp(c * scale) = 2^(c * s2) with s2 = scale * log2(e) (decoder.py:57-63), in float32 (the code
// as a float by the 2^23 bias trick, one ex2 per pair).  The (cos, sin) of the 8-bit angle code
// come from a 256-entry float2 table held 16 times, copy j at float2 index 16 * c + j: lane l
// reads copy l % 16, so each half warp's 64-bit lookups hit 16 different bank pairs.
__device__ __forceinline__ void decode_row_adapter(const uint8_t* stage, const AttnParams& P, const float2* tab,
                                                   float s2, int r, int t, uint32_t (&kp)[16]) {
  const uint4 R = lds128(stage + r * kPairs + 16 * t);
  const uint4 C = lds128(stage + P.off_codes + r * kPairs + 16 * t);
  // Radius codes as unsigned bytes c + 128 (two's complement with the sign bit flipped).
  const uint32_t rw[4] = {R.x ^ 0x80808080u, R.y ^ 0x80808080u, R.z ^ 0x80808080u, R.w ^ 0x80808080u};
  const uint32_t cw[4] = {C.x, C.y, C.z, C.w};
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    // 0x4B0000xx is the float 2^23 + xx: minus 2^23 + 128 leaves the signed code exactly.
    const float code = __uint_as_float(prmt(rw[i >> 2], 0x4B000000u, 0x7540u | uint32_t(i & 3))) - 8388736.f;
    const float rad = exp2_approx(code * s2);
    const uint32_t c = prmt(cw[i >> 2], 0u, 0x4440u | uint32_t(i & 3));
    const float2 a = tab[c << 4];
    kp[i] = pack_h2(rad * a.x, rad * a.y);
  }
}

// Key decode of a page pass: the general path (any format), the table-driven default format,
// and the adapter format.
enum { kModeGeneral = 0, kModeFast = 1, kModeAdapter = 2 };

// ----------------------------------------------------------------------------- one half page
// TP_QK_CUDA_CORES: float offset of key pair j's 4 query heads (float2 each) in a warp's query
// copy, 4 floats of padding per 16 pairs so the 4 lanes of a quad hit different banks.
__device__ __forceinline__ int qcc_off(int j) { return j * 8 + (j >> 4) * 4; }
constexpr int kQccFloats = 528;

// Formats whose P.V is exact: the TP_EXACT_PV key formats, and every format with dense values.
template <int kMode, bool kDenseV>
__host__ __device__ constexpr bool exact_pv() {
  return kDenseV || ((TP_EXACT_PV >> kMode) & 1);
}

template <int kMode, bool kDenseV>
__device__ __forceinline__ void process_half(WarpAcc& A, const uint8_t* stage, const AttnParams& P, const float2* lut,
                                             const float2* tab, const uint32_t (&qf)[16], float radius_scale,
                                             int valid_tokens, int lane
#if TP_QK_CUDA_CORES
                                             , const float* qs
#endif
                                             ) {
  const int g = lane >> 2, t = lane & 3;
  float sc[2][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    uint32_t k0[16], k1[16];
    if (kMode == kModeFast) {
      const uint32_t tab_sa = (smem_u32(lut) + 255u) & ~255u;
      decode_row_fast(stage, P, tab_sa, 16 * mt + g, t, k0);
      decode_row_fast(stage, P, tab_sa, 16 * mt + g + 8, t, k1);
    } else if (kMode == kModeAdapter) {
      decode_row_adapter(stage, P, tab, radius_scale, 16 * mt + g, t, k0);
      decode_row_adapter(stage, P, tab, radius_scale, 16 * mt + g + 8, t, k1);
    } else {
      decode_row_general(stage, P, lut, radius_scale, 16 * mt + g, t, k0);
      decode_row_general(stage, P, lut, radius_scale, 16 * mt + g + 8, t, k1);
    }
#if TP_QK_CUDA_CORES
    if (kMode == kModeFast) {
      float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int j = 16 * t + i;
        const float4 qa = *reinterpret_cast<const float4*>(qs + qcc_off(j));
        const float4 qb = *reinterpret_cast<const float4*>(qs + qcc_off(j) + 4);
        const float2 ka = __half22float2(u32_as_h2(k0[i])), kb = __half22float2(u32_as_h2(k1[i]));
        s0[0] = fmaf(ka.x, qa.x, fmaf(ka.y, qa.y, s0[0])); s0[1] = fmaf(ka.x, qa.z, fmaf(ka.y, qa.w, s0[1]));
        s0[2] = fmaf(ka.x, qb.x, fmaf(ka.y, qb.y, s0[2])); s0[3] = fmaf(ka.x, qb.z, fmaf(ka.y, qb.w, s0[3]));
        s1[0] = fmaf(kb.x, qa.x, fmaf(kb.y, qa.y, s1[0])); s1[1] = fmaf(kb.x, qa.z, fmaf(kb.y, qa.w, s1[1]));
        s1[2] = fmaf(kb.x, qb.x, fmaf(kb.y, qb.y, s1[2])); s1[3] = fmaf(kb.x, qb.z, fmaf(kb.y, qb.w, s1[3]));
      }
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        s0[h] += __shfl_xor_sync(0xffffffffu, s0[h], 1);
        s0[h] += __shfl_xor_sync(0xffffffffu, s0[h], 2);
        s1[h] += __shfl_xor_sync(0xffffffffu, s1[h], 1);
        s1[h] += __shfl_xor_sync(0xffffffffu, s1[h], 2);
      }
      // The mma accumulator layout: rows g, g + 8; heads 2t, 2t + 1 (heads >= 4 are zero).
      sc[mt][0] = t == 0 ? s0[0] : (t == 1 ? s0[2] : 0.f);
      sc[mt][1] = t == 0 ? s0[1] : (t == 1 ? s0[3] : 0.f);
      sc[mt][2] = t == 0 ? s1[0] : (t == 1 ? s1[2] : 0.f);
      sc[mt][3] = t == 0 ? s1[1] : (t == 1 ? s1[3] : 0.f);
      continue;
    }
#endif
    float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < 8; ks += 2) {
      mma16816(a0, k0[2 * ks], k1[2 * ks], k0[2 * ks + 1], k1[2 * ks + 1], qf[2 * ks], qf[2 * ks + 1]);
      mma16816(a1, k0[2 * ks + 2], k1[2 * ks + 2], k0[2 * ks + 3], k1[2 * ks + 3], qf[2 * ks + 2], qf[2 * ks + 3]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) sc[mt][j] = a0[j] + a1[j];
  }
  if (valid_tokens < kHalf) {
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      if (16 * mt + g >= valid_tokens) sc[mt][0] = sc[mt][1] = -INFINITY;
      if (16 * mt + g + 8 >= valid_tokens) sc[mt][2] = sc[mt][3] = -INFINITY;
    }
  }
  constexpr bool kExact = exact_pv<kMode, kDenseV>();
  softmax_update<2, !kExact>(A, sc, P.scale_log2);
  if (kDenseV) {
    // Tile 2G (2G+1) rows g, g + 8 are channels d0, d0 + 1 (d0 + 2, d0 + 3), d0 = 32G + 4g, as
    // the code path's tiles (store_warp_partial).  Lane (g, t) reads 8 bytes (channels d0 ..
    // d0 + 3) of tokens 2t, 2t + 1, 2t + 8, 2t + 9 of the 16-token tile: in box G / 2 at chunk
    // 4(G & 1) + g / 2, byte 8(g & 1); with the chunk swizzled by the token row, the 16 lanes of
    // a half warp read 16 different 8-byte bank pairs.  One byte permute then pairs the two
    // tokens of a fragment register.
    const uint8_t* vd = stage + P.off_vdense;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const uint32_t h0 = pack_h2(sc[mt][0], sc[mt][1]), h1 = pack_h2(sc[mt][2], sc[mt][3]);
      const float2 f0 = __half22float2(u32_as_h2(h0)), f1 = __half22float2(u32_as_h2(h1));
      const uint32_t bh0 = movmatrix_trans(h0), bh1 = movmatrix_trans(h1);
      const uint32_t bl0 = movmatrix_trans(pack_h2(sc[mt][0] - f0.x, sc[mt][1] - f0.y));
      const uint32_t bl1 = movmatrix_trans(pack_h2(sc[mt][2] - f1.x, sc[mt][3] - f1.y));
      const int r0 = 16 * mt + 2 * t;
#pragma unroll
      for (int G = 0; G < 4; ++G) {
        const uint8_t* box = vd + (G >> 1) * 4096 + 8 * (g & 1);
        const int ch = 4 * (G & 1) + (g >> 1);
        auto row = [&](int r) { return lds64(box + r * 128 + ((ch ^ (r & 7)) << 4)); };
        const uint2 x0 = row(r0), x1 = row(r0 + 1), x8 = row(r0 + 8), x9 = row(r0 + 9);
        const uint32_t a0 = prmt(x0.x, x1.x, 0x5410), a1 = prmt(x0.x, x1.x, 0x7632);
        const uint32_t a2 = prmt(x8.x, x9.x, 0x5410), a3 = prmt(x8.x, x9.x, 0x7632);
        mma16816(A.o[2 * G], a0, a1, a2, a3, bh0, bh1);
        mma16816(A.o[2 * G], a0, a1, a2, a3, bl0, bl1);
        const uint32_t c0 = prmt(x0.y, x1.y, 0x5410), c1 = prmt(x0.y, x1.y, 0x7632);
        const uint32_t c2 = prmt(x8.y, x9.y, 0x5410), c3 = prmt(x8.y, x9.y, 0x7632);
        mma16816(A.o[2 * G + 1], c0, c1, c2, c3, bh0, bh1);
        mma16816(A.o[2 * G + 1], c0, c1, c2, c3, bl0, bl1);
      }
    }
    return;
  }
  const uint8_t* vcodes = stage + P.off_vcodes;
  const uint8_t* vscales = stage + P.off_vscales;
  const uint32_t K = 0x64646464u;  // float16 0x64xx = 1024 + xx: a byte permute makes code + 1152
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    // (scale[tok][G], scale[tok+1][G]) for this lane's token pairs (2t, 2t+1) and (2t+8, 2t+9).
    const uint4 S01 = lds128(vscales + mt * 128 + t * 32);
    const uint4 S89 = lds128(vscales + mt * 128 + t * 32 + 16);
    const uint32_t s01[4] = {S01.x, S01.y, S01.z, S01.w}, s89[4] = {S89.x, S89.y, S89.z, S89.w};
    if (kExact) {
      // Exact P.V.  V is dequantised on the A side as the reference dequantises it
      // (v_quant/encoder.py:32-38: fp16(code * scale)): the biased code minus 1152 is the code
      // exactly, and one float16 multiply by the token's scale rounds once.  P enters as float16
      // hi + lo parts (hi = fp16(p), lo = fp16(p - hi)), two products per tile, so the weights
      // carry about 22 bits; no bias tile is needed.
      const uint32_t h0 = pack_h2(sc[mt][0], sc[mt][1]), h1 = pack_h2(sc[mt][2], sc[mt][3]);
      const float2 f0 = __half22float2(u32_as_h2(h0)), f1 = __half22float2(u32_as_h2(h1));
      const uint32_t bh0 = movmatrix_trans(h0), bh1 = movmatrix_trans(h1);
      const uint32_t bl0 = movmatrix_trans(pack_h2(sc[mt][0] - f0.x, sc[mt][1] - f0.y));
      const uint32_t bl1 = movmatrix_trans(pack_h2(sc[mt][2] - f1.x, sc[mt][3] - f1.y));
      const uint32_t kBias = 0x64806480u;  // float16 1152 in both halves
#pragma unroll
      for (int G = 0; G < 4; ++G) {
        const uint4 W = lds128(vcodes + mt * 2048 + G * 512 + lane * 16);
        auto dq = [&](uint32_t w, uint32_t sel, uint32_t sc2) {
          return hmul2u(h2_as_u32(__hsub2(u32_as_h2(prmt(w, K, sel)), u32_as_h2(kBias))), sc2);
        };
        const uint32_t a0 = dq(W.x, 0x4140, s01[G]), a1 = dq(W.x, 0x4342, s01[G]);
        const uint32_t a2 = dq(W.z, 0x4140, s89[G]), a3 = dq(W.z, 0x4342, s89[G]);
        mma16816(A.o[2 * G], a0, a1, a2, a3, bh0, bh1);
        mma16816(A.o[2 * G], a0, a1, a2, a3, bl0, bl1);
        const uint32_t c0 = dq(W.y, 0x4140, s01[G]), c1 = dq(W.y, 0x4342, s01[G]);
        const uint32_t c2 = dq(W.w, 0x4140, s89[G]), c3 = dq(W.w, 0x4342, s89[G]);
        mma16816(A.o[2 * G + 1], c0, c1, c2, c3, bh0, bh1);
        mma16816(A.o[2 * G + 1], c0, c1, c2, c3, bl0, bl1);
      }
      continue;
    }
    const uint32_t kOne = 0x3C003C00u;
    const uint32_t b0 = movmatrix_trans(pack_h2(sc[mt][0], sc[mt][1]));
    const uint32_t b1 = movmatrix_trans(pack_h2(sc[mt][2], sc[mt][3]));
#pragma unroll
    for (int G = 0; G < 4; ++G) {
      const uint32_t bg0 = hmul2u(b0, s01[G]), bg1 = hmul2u(b1, s89[G]);
      // Biased codes of this lane's A fragments for tiles 2G and 2G+1, token pairs interleaved.
      const uint4 W = lds128(vcodes + mt * 2048 + G * 512 + lane * 16);
      mma16816(A.o[2 * G], prmt(W.x, K, 0x4140), prmt(W.x, K, 0x4342), prmt(W.z, K, 0x4140), prmt(W.z, K, 0x4342), bg0, bg1);
      mma16816(A.o[2 * G + 1], prmt(W.y, K, 0x4140), prmt(W.y, K, 0x4342), prmt(W.w, K, 0x4140), prmt(W.w, K, 0x4342), bg0, bg1);
      mma16816(A.ones[G], kOne, kOne, kOne, kOne, bg0, bg1);
    }
  }
}

// ----------------------------------------------------------------------------- staging
// Unit `half` of page `page` of KV head kvh into a stage: one bulk copy (every unit is
// contiguous in the pool) completing on the stage's mbarrier.
__device__ __forceinline__ void issue_half(uint8_t* stage, uint64_t* bar, const AttnParams& P, int kvh, int page,
                                           int half, int part, uint64_t pol) {
  const int64_t unit = (int64_t(kvh) * P.page_capacity + page) * 2 + half;
  const int chunk = (P.unit_bytes / kCopySplit + 15) & ~15;
  const int off = min(part * chunk, P.unit_bytes);
  const uint32_t bytes = uint32_t(min(chunk, P.unit_bytes - off));
  fence_proxy_async_smem();
  mbar_arrive_expect_tx(bar, bytes);
  if (bytes) bulk_g2s_hint(stage + off, P.pages + unit * P.unit_bytes + off, bytes, bar, pol);
}

// Dense-V variant: the unit's radii and angle codes (bulk copies) and the 32 value rows of its
// tokens (page * 64 + half * 32 of KV head kvh in the value array; two TMA boxes), all by part
// 0; the other parts only arrive.
__device__ __forceinline__ void issue_half_dense_v(uint8_t* stage, uint64_t* bar, const AttnParams& P, int kvh,
                                                   int page, int half, int part, uint64_t pol) {
  if (part != 0) {
    mbar_arrive(bar);
    return;
  }
  const int64_t unit = (int64_t(kvh) * P.page_capacity + page) * 2 + half;
  const uint8_t* src = P.pages + unit * P.unit_bytes;
  const int tok = page * kPage + half * kHalf;
  fence_proxy_async_smem();
  mbar_arrive_expect_tx(bar, uint32_t(P.k_radii_bytes + P.k_code_bytes + 2 * kHalf * 64 * 2));
  bulk_g2s_hint(stage, src, uint32_t(P.k_radii_bytes), bar, pol);
  bulk_g2s_hint(stage + P.off_codes, src + P.k_src_codes, uint32_t(P.k_code_bytes), bar, pol);
  tma_load_3d(stage + P.off_vdense, &P.vmap, 0, tok, kvh, bar, pol);
  tma_load_3d(stage + P.off_vdense + 4096, &P.vmap, 64, tok, kvh, bar, pol);
}

// Bounded wait for phase `parity` of a stage barrier (about a second); false on timeout.
__device__ __forceinline__ bool stage_wait(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > (1ll << 31)) return false;
  }
  return true;
}

__device__ __forceinline__ void load_q_frags(const AttnParams& P, int qh_base, int gc, int lane, uint32_t (&qf)[16]) {
  const int g = lane >> 2, t = lane & 3;
  if (g < gc) {
    const int64_t row = int64_t(qh_base + g) * kD + 32 * t;
    if (P.q_f32) {
      const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(P.q) + row);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 v = p[i];
        qf[2 * i] = pack_h2(v.x, v.y);
        qf[2 * i + 1] = pack_h2(v.z, v.w);
      }
    } else {
      const uint4* p = reinterpret_cast<const uint4*>(static_cast<const __half*>(P.q) + row);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 v = p[i];
        qf[4 * i] = v.x; qf[4 * i + 1] = v.y; qf[4 * i + 2] = v.z; qf[4 * i + 3] = v.w;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) qf[i] = 0u;
  }
}

// Write this warp's partial (m, l, o) for the heads < gc to a record of kHeadStride floats a
// head ([gc][130] in shared memory; [gc][132] in the workspace, 16-byte aligned heads).
template <bool kExact, int kHeadStride = TP_PARTIAL_FLOATS>
__device__ __forceinline__ void store_warp_partial(WarpAcc& A, float* rec, int gc, int lane) {
  const int g = lane >> 2, t = lane & 3;
  float l0 = A.l[0], l1 = A.l[1];
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  const int h0 = 2 * t, h1 = 2 * t + 1;
#pragma unroll
  for (int md = 0; md < 8; ++md) {
    const int G = md >> 1;
    const int d = 32 * G + 4 * g + 2 * (md & 1);
    const float c0 = kExact ? 0.f : 1152.f * A.ones[G][0], c1 = kExact ? 0.f : 1152.f * A.ones[G][1];
    if (h0 < gc) {
      rec[h0 * kHeadStride + 2 + d] = A.o[md][0] - c0;
      rec[h0 * kHeadStride + 3 + d] = A.o[md][2] - c0;
    }
    if (h1 < gc) {
      rec[h1 * kHeadStride + 2 + d] = A.o[md][1] - c1;
      rec[h1 * kHeadStride + 3 + d] = A.o[md][3] - c1;
    }
  }
  if (g == 0) {
    if (h0 < gc) { rec[h0 * kHeadStride] = A.m[0]; rec[h0 * kHeadStride + 1] = l0; }
    if (h1 < gc) { rec[h1 * kHeadStride] = A.m[1]; rec[h1 * kHeadStride + 1] = l1; }
  }
}

template <int kHeadStride = TP_PARTIAL_FLOATS>
__device__ __forceinline__ void store_empty_partial(float* rec, int gc, int lane) {
  for (int i = lane; i < gc * kHeadStride; i += 32) rec[i] = (i % kHeadStride == 0) ? -INFINITY : 0.f;
}

// Final write of one head's merged (m, l, o[d]).
__device__ __forceinline__ void write_result(const AttnParams& P, int qh, int d, float m, float l, float o) {
  if (P.partial_out) {
    float* rec = P.partial_out + int64_t(qh) * TP_PARTIAL_FLOATS;
    if (d == 0) { rec[0] = m; rec[1] = l; }
    rec[2 + d] = o;
  } else {
    P.out[int64_t(qh) * kD + d] = __float2half_rn(l > 0.f ? o / l : 0.f);
  }
}

// ----------------------------------------------------------------------------- kernel
__device__ __forceinline__ tp_state read_state(const AttnParams& P) {
  tp_state st = P.st;
  if (P.d_state) {
    st.n_pages = P.d_state[0];
    st.tail_len = P.d_state[1];
    st.seq_len = P.d_state[2];
    st.first_page = P.d_state[3];
  }
  return st;
}

// This CTA's share of the page pass: units (half pages, head-major) [u0, u1) spanning at most
// two heads ("segments"): n units, the first n0 of segment 0 (head vh_first) starting at its
// unit a0, the rest of segment 1 starting at its unit 0.  Whole-segment partition (kOwner, more
// segments than CTAs): segments [vh_first, vh_first + nseg), all of their units.
struct Part {
  int n_pages;
  bool active;
  int vh_first, nseg, n, n0, a0;
};

template <bool kOwner>
__device__ __forceinline__ Part make_part(const AttnParams& P, const tp_state& st, int c) {
  Part pt = {};
  pt.n_pages = min(max(st.n_pages, 0), P.page_capacity);
  if (kOwner) {
    // CTA c owns segments [floor(c*V/G), floor((c+1)*V/G)), V = k*G + r as in part_begin.
    Grid g;
    g.U = P.num_kv_heads * P.nqc;
    g.C = int(gridDim.x);
    g.k = g.U / g.C;
    g.r = g.U - g.k * g.C;
    pt.vh_first = part_begin(g, c);
    pt.nseg = part_begin(g, c + 1) - pt.vh_first;
    pt.active = pt.n_pages > 0 && pt.nseg > 0;
    pt.n = pt.nseg * 2 * pt.n_pages;
    pt.n0 = 2 * pt.n_pages;
    pt.a0 = 0;
    return pt;
  }
  const Grid g = grid_of(P.num_kv_heads * P.nqc, pt.n_pages, int(gridDim.x));
  const int uph = g.uph;
  pt.active = g.U > 0 && c < g.C;
  if (!pt.active) return pt;
  const int u0 = part_begin(g, c), u1 = part_begin(g, c + 1);
  pt.vh_first = u0 / uph;
  pt.nseg = (u1 - 1) / uph - pt.vh_first + 1;
  const int hb0 = pt.vh_first * uph;
  pt.n = u1 - u0;
  pt.n0 = min(u1, hb0 + uph) - u0;
  pt.a0 = u0 - hb0;
  return pt;
}

// Segment, page and half of CTA unit k.
__device__ __forceinline__ int3 unit_ref(const Part& pt, int k) {
  const int seg = k >= pt.n0 ? 1 : 0;
  const int j = seg ? k - pt.n0 : pt.a0 + k;
  return make_int3(seg, j >> 1, j & 1);
}

// Bounded wait for the producer (false on timeout).
__device__ __forceinline__ bool slot_wait(uint64_t* bar, uint32_t parity) { return stage_wait(bar, parity); }

// Page pass.  Warps 0..kConsumers-1 compute; the kProducerWarps warps after them copy.
// Consumer w takes CTA units w, w + kConsumers, ... and owns ring stages [w*S, w*S + S)
// (S = P.n_stages / kConsumers), its j-th unit in stage w*S + j % S; each stage has a "full"
// mbarrier (the bulk copy of a unit completes on it) and an "empty" one (the consumer releases
// the stage).  Issuing lane p of the copy warp(s) serves consumer p / kCopySplit: it issues
// part p % kCopySplit of each of that consumer's units in turn (one bulk copy; the stage's
// full barrier expects kCopySplit arrivals), waiting for the stage's release before reusing
// it.  Every stage is filled and drained by fixed threads that follow its phases in order, so
// no wait is ever more than one phase ahead of its barrier.  A thread dispatches one bulk copy
// at a time, so the copies are spread over lanes that never hold up the warps that compute;
// consumers get the same number of units to within one.
// At most 192 registers a thread: 8 warps of the page pass and 8 of a combine kernel (48 or 64
// each) then fit the SM's 64K registers together (the CUDA-core comparison variant needs more).
#if TP_QK_CUDA_CORES
#define TP_PAGE_PASS_REGS 255
#else
#define TP_PAGE_PASS_REGS 192
#endif
template <int kMode, bool kDenseV, bool kOwner>
__global__ void __maxnreg__(TP_PAGE_PASS_REGS) decode_attention_kernel(const __grid_constant__ AttnParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr bool kExactPV = exact_pv<kMode, kDenseV>();
  __shared__ tp_state s_pre;  // cache state as read before the wait, one read for the CTA
  __shared__ float s_wt[2][kMaxHeads][kConsumers + 1];  // merge weights, then the maximum
  float2* lut = reinterpret_cast<float2*>(smem + P.smem_lut_off);
  float* merge = reinterpret_cast<float*>(smem + P.smem_merge_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + P.smem_bar_off);
  uint64_t* empty = full + kMaxStages;
  uint8_t* ring = smem + P.smem_stage_off;
  // Dense values: the swizzled TMA boxes need 1024-byte aligned shared addresses (the host
  // reserves 1024 bytes for this).
  if (kDenseV) ring += (1024u - (smem_u32(ring) & 1023u)) & 1023u;
  float* stage_scale = reinterpret_cast<float*>(smem + P.smem_scale_off);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int R = P.n_stages, S = R / kConsumers;
  const int gmax = P.gmax;
  const int rec_stride = gmax * TP_PARTIAL_FLOATS;
  const bool producer = warp >= kConsumers;
  const int pw = (warp - kConsumers) * 32 + lane;  // issuing-lane index
  const bool issuer = producer && pw < kIssuers;
  const int pcons = pw / kCopySplit, ppart = pw % kCopySplit;  // the consumer and part it serves
  const int c = blockIdx.x;
  const uint64_t pol = l2_evict_first_policy();
  if (kDenseV && issuer && pw == 0) prefetch_tmap(&P.vmap);

  // Before the previous kernel in the stream has completed (this grid is its programmatic
  // dependent): the code tables, the ring barriers and the first copies, none of which
  // depends on anything that kernel writes.
  if (kMode == kModeAdapter) {
    // Entry c of the deep table, 16 copies (float2 index 16 * c + j): a warp-uniform parameter
    // load, stored by lanes 0-15.
    float2* tab = reinterpret_cast<float2*>(smem + P.smem_tab_off);
    for (int c = warp; c < kLutEntries; c += kThreads / 32) {
      const float2 v = P.cs[c];
      if (lane < 16) tab[16 * c + lane] = v;
    }
  } else if (kMode == kModeFast) {
    if (tid < 16) {  // at the first 256-byte boundary of the table region (256 bytes of slack)
      const uint32_t sa = (smem_u32(lut) + 255u) & ~255u;
      reinterpret_cast<float2*>(reinterpret_cast<uint8_t*>(lut) + (sa - smem_u32(lut)))[tid] = P.cs[tid];
    }
  } else {
    const int n1 = 1 << P.l1_bits, n2 = 1 << P.deep_bits;
    for (int i = tid; i < n1 + n2; i += kThreads)
      lut[i] = i < n1 ? cos_sin_of_code(i, P.l1_bits) : cos_sin_of_code(i - n1, P.deep_bits);
  }
  auto init_barriers = [&]() {
    for (int st = 0; st < R; ++st) {
      mbar_init(&full[st], kCopySplit);
      mbar_init(&empty[st], 1);
    }
    fence_mbar_init();
  };
  if (tid == 0) {
    const tp_state st0 = read_state(P);  // loads in flight while the barriers are set up
    init_barriers();
    s_pre = st0;
  }
  __syncthreads();  // barriers initialised and the state read before any producer issues
  Part pt = make_part<kOwner>(P, s_pre, c);
  bool timed_out = false;
  // Units of consumer w, and its q-th unit as (segment, page, half): CTA units w, w + kConsumers,
  // ... of the CTA's unit list (the whole-segment partition's list runs through its segments one
  // after another).
  auto units_of = [&](int w) { return pt.n > w ? (pt.n - 1 - w) / kConsumers + 1 : 0; };
  auto unit_at = [&](int w, int q) {
    if (kOwner) {
      const int k = w + kConsumers * q, uph = 2 * pt.n_pages, seg = k / uph, j = k - seg * uph;
      return make_int3(seg, j >> 1, j & 1);
    }
    return unit_ref(pt, w + kConsumers * q);
  };
  // Issue the j-th unit of consumer w (issuing lanes only).  After a release wait runs out
  // nothing more is issued (the consumers' own bounded waits then run out and return).
  auto produce = [&](int w, int j) {
    const int slot = w * S + j % S, wrap = j / S;
    if (wrap > 0 && !stage_wait(&empty[slot], uint32_t(wrap - 1) & 1u)) {
      timed_out = true;
      return;
    }
    const int3 u = unit_at(w, j);
    const int kvh = (pt.vh_first + u.x) / P.nqc;
    // The unit's radius scale travels beside its copy: stored before the arrival on the
    // stage's full barrier, which releases it to the consumer.
    if (P.int8_radii && ppart == 0)
      stage_scale[slot] = __half2float(P.radii_scales[int64_t(kvh) * P.page_capacity + u.y]);
    if (kDenseV) issue_half_dense_v(ring + slot * P.stage_bytes, &full[slot], P, kvh, u.y, u.z, ppart, pol);
    else issue_half(ring + slot * P.stage_bytes, &full[slot], P, kvh, u.y, u.z, ppart, pol);
  };
  // Units [j0, j1) of the consumer this lane serves.
  auto produce_range = [&](int j0, int j1) {
    const int nu = units_of(pcons);
    for (int j = j0; j < j1 && j < nu && !timed_out; ++j) produce(pcons, j);
  };
  bool early = false;
  tp_state st = s_pre;
  if (P.spec) {
    // The previous kernel in the stream writes nothing this launch reads (the host compared
    // the two calls' buffers), so the state read above is final and the whole pass runs
    // now; the wait comes before the partials are written (the workspace may be shared with
    // the previous call, whose split combine reads its own partials until it completes).  The
    // split-combine grid may become resident at once.
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  } else {
    // Each consumer's first S units go in flight now, on the partition of the page count read
    // now.  Every page below the newest one was written by a launch that had completed before
    // the previous kernel in the stream started, so copies of those are valid whatever that
    // kernel does; the newest page may be the one it is writing (an append that completed a
    // page), so nothing is issued early if the first units touch it -- unless no call that
    // may still run writes this cache (P.cache_final), when the state read above is final too.
    early = pt.active;
    for (int w = 0; early && !P.cache_final && w < kConsumers; ++w)
      for (int q = 0; early && q < min(S, units_of(w)); ++q) early = unit_at(w, q).y < pt.n_pages - 1;
    if (early && issuer) produce_range(0, S);

    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    // Let the split-combine grid become resident now; it waits for this grid to complete.
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    if (!P.cache_final) st = read_state(P);
  }
  if (!P.spec && min(max(st.n_pages, 0), P.page_capacity) != pt.n_pages) {
    // The previous kernel appended to this cache: let the early copies land, reset the
    // barriers and start again on the new partition.
    if (early && issuer) {
      for (int j = 0; j < S; ++j)
        if (j < units_of(pcons) && !stage_wait(&full[pcons * S + j], 0)) timed_out = true;
    }
    __syncthreads();
    if (tid == 0) {
      for (int i = 0; i < R; ++i) {
        mbar_inval(&full[i]);
        mbar_inval(&empty[i]);
      }
      init_barriers();
    }
    early = false;
    pt = make_part<kOwner>(P, st, c);
  }
  __syncthreads();  // code tables; barriers reset if the partition changed
  if (!pt.active) {
    if (timed_out) atomicExch(P.ws_error, 1);
    // The grid's completion must imply the previous kernel's (a later call that waits for this
    // call relies on it), also when no CTA has a unit.
    if (P.spec) asm volatile("griddepcontrol.wait;\n" ::: "memory");
    return;
  }
  const int n = pt.n, nseg = pt.nseg, vh_first = pt.vh_first;

  if (producer) {
    if (issuer) {
      produce_range(early ? S : 0, units_of(pcons));
      if (timed_out) atomicExch(P.ws_error, 1);  // word 0: 1 after a wait ran out
    }
  } else {
    WarpAcc A;
    uint32_t qf[16];
    const float2* tab = reinterpret_cast<const float2*>(smem + P.smem_tab_off) + (lane & 15);
#if TP_QK_CUDA_CORES
    float* qcc = reinterpret_cast<float*>(smem + P.smem_qcc_off) + warp * kQccFloats;
#endif
    int cur = -1;        // segment of the accumulator (-1: none yet)
    int kvh = 0, gc = gmax;
    // Ring stage and phase of this warp's next unit.
    int js = 0, wrap = 0;
    // One unit of the ring: wait for its copy, attend, release the stage.
    auto consume = [&](int page, int half) {
      const int slot = warp * S + js;
      const bool ready = stage_wait(&full[slot], uint32_t(wrap) & 1u);
      if (ready) {
        const int64_t pos0 = (int64_t(st.first_page) + page) * kPage + half * kHalf;
        const int vt = int(clamp64(int64_t(st.seq_len) - pos0, 0, kHalf));
        // The adapter path takes the radius scale in base-2 units.
        const float rs = P.int8_radii ? stage_scale[slot] * (kMode == kModeAdapter ? 1.4426950408889634f : 1.f) : 0.f;
        process_half<kMode, kDenseV>(A, ring + slot * P.stage_bytes, P, lut, tab, qf, rs, vt, lane
#if TP_QK_CUDA_CORES
                                     , qcc
#endif
        );
      } else {
        timed_out = true;  // the unit is left out; the error word marks the result unusable
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (++js == S) { js = 0; ++wrap; }
    };
    if (kOwner) {
      // Whole segments.  The warp's units run through the CTA's segments one after another; at
      // every change of segment it writes its partial of the segment it leaves to that segment's
      // workspace record of this warp, (segment * kConsumers + warp), and an empty record for
      // every segment it has no unit of, so the split combine finds kConsumers records per
      // segment.  Nothing here waits for the other warps.
      const int uph = 2 * pt.n_pages;
      bool waited = !P.spec || P.ws_private;  // the workspace may be the previous call's (see below)
      auto rec_of = [&](int sl) {
        return P.ws_partials + (int64_t(vh_first + sl) * kConsumers + warp) * kPartialStride;
      };
      auto before_store = [&]() {
        if (!waited) {  // the previous call's split combine reads its records until it completes
          asm volatile("griddepcontrol.wait;\n" ::: "memory");
          waited = true;
        }
      };
      cur = -1;
      for (int k = warp; k < n; k += kConsumers) {
        const int sl = k / uph, j = k - sl * uph;
        if (sl != cur) {
          before_store();
          if (cur >= 0) store_warp_partial<kExactPV, kRecFloats>(A, rec_of(cur), gc, lane);
          for (int e = cur + 1; e < sl; ++e) store_empty_partial<kRecFloats>(rec_of(e), gmax, lane);
          cur = sl;
          const int vh = vh_first + sl, chunk = vh % P.nqc;
          kvh = vh / P.nqc;
          gc = min(kMaxHeads, P.group - chunk * kMaxHeads);
          load_q_frags(P, kvh * P.group + chunk * kMaxHeads, gc, lane, qf);
          acc_reset(A);
        }
        consume(j >> 1, j & 1);
      }
      before_store();
      if (cur >= 0) store_warp_partial<kExactPV, kRecFloats>(A, rec_of(cur), gc, lane);
      for (int e = cur + 1; e < nseg; ++e) store_empty_partial<kRecFloats>(rec_of(e), gmax, lane);
      if (timed_out && lane == 0) atomicExch(P.ws_error, 1);  // word 0: 1 after a stage-wait timeout
    } else {
    for (int k = warp; k < n; k += kConsumers) {
      const int3 u = unit_ref(pt, k);
      if (u.x != cur) {
        if (cur == 0) store_warp_partial<kExactPV>(A, merge + warp * rec_stride, gc, lane);
        else if (u.x == 1) store_empty_partial(merge + warp * rec_stride, gmax, lane);
        cur = u.x;
        const int vh = vh_first + cur, chunk = vh % P.nqc;
        kvh = vh / P.nqc;
        gc = min(kMaxHeads, P.group - chunk * kMaxHeads);
        load_q_frags(P, kvh * P.group + chunk * kMaxHeads, gc, lane, qf);
#if TP_QK_CUDA_CORES
        {  // float32 copy of the chunk's query heads for the CUDA-core Q.K
          const int qh0 = kvh * P.group + chunk * kMaxHeads;
          for (int jj = lane; jj < kPairs; jj += 32)
            for (int h = 0; h < 4; ++h) {
              float2 v = make_float2(0.f, 0.f);
              if (h < gc) {
                const __half* qp = static_cast<const __half*>(P.q) + int64_t(qh0 + h) * kD + 2 * jj;
                v = make_float2(__half2float(qp[0]), __half2float(qp[1]));
              }
              *reinterpret_cast<float2*>(qcc + qcc_off(jj) + 2 * h) = v;
            }
          __syncwarp();
        }
#endif
        acc_reset(A);
      }
      consume(u.y, u.z);
    }
    // Segment 0 partials go to the merge region now; segment 1 partials to this warp's ring
    // stage once every consumer is done with the ring (all issued copies have landed).
    if (cur == 0) store_warp_partial<kExactPV>(A, merge + warp * rec_stride, gc, lane);
    else if (cur == -1) store_empty_partial(merge + warp * rec_stride, gmax, lane);
    if (timed_out && lane == 0) atomicExch(P.ws_error, 1);  // word 0: 1 after a stage-wait timeout
    asm volatile("bar.sync 1, %0;\n" ::"n"(kConsumers * 32) : "memory");
    if (nseg > 1) {
      float* rec1 = reinterpret_cast<float*>(ring + warp * P.stage_bytes);
      if (cur == 1) store_warp_partial<kExactPV>(A, rec1, gc, lane);
      else store_empty_partial(rec1, gmax, lane);
    }
    }
  }
  if (P.spec && !P.ws_private) asm volatile("griddepcontrol.wait;\n" ::: "memory");
  __syncthreads();
  if (kOwner) {  // every segment's record is written
    if (P.spec && P.ws_private) asm volatile("griddepcontrol.wait;\n" ::: "memory");
    return;
  }

  // Merge the warps of each segment and publish this CTA's partial; the split-combine kernel
  // (launched as a programmatic dependent of this grid) merges the CTAs of every head.  The
  // weight of warp w's partial for head h, exp2(m_w - M_h), is computed once per (segment,
  // head, warp) and read by every channel.
  auto seg_recs = [&](int s) { return s == 0 ? merge : reinterpret_cast<const float*>(ring); };
  auto seg_stride = [&](int s) { return s == 0 ? rec_stride : P.stage_bytes / int(sizeof(float)); };
  for (int i = tid; i < nseg * gmax * kConsumers; i += kThreads) {
    const int s = i / (gmax * kConsumers), h = (i / kConsumers) % gmax, w = i % kConsumers;
    const float* recs = seg_recs(s) + h * TP_PARTIAL_FLOATS;
    const int wstride = seg_stride(s);
    float M = recs[0];
#pragma unroll
    for (int v = 1; v < kConsumers; ++v) M = fmaxf(M, recs[v * wstride]);
    const float m = recs[w * wstride];
    s_wt[s][h][w] = (m == -INFINITY) ? 0.f : exp2_approx(m - M);
    if (w == 0) s_wt[s][h][kConsumers] = M;
  }
  __syncthreads();
  for (int s = 0; s < nseg; ++s) {
    const int vh = vh_first + s;
    const int chunk = vh % P.nqc;
    const int gc = min(kMaxHeads, P.group - chunk * kMaxHeads);
    float* slot = P.ws_partials + int64_t(c * 2 + s) * kPartialStride;
    const float* recs = seg_recs(s);
    const int wstride = seg_stride(s);
#pragma unroll 1
    for (int i = tid; i < gc * kD; i += kThreads) {
      const int h = i >> 7, d = i & (kD - 1);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) {
        const float* r = recs + w * wstride + h * TP_PARTIAL_FLOATS;
        const float f = s_wt[s][h][w];
        L = fmaf(r[1], f, L);
        O = fmaf(r[2 + d], f, O);
      }
      float* out = slot + h * kRecFloats;
      if (d == 0) { out[0] = s_wt[s][h][kConsumers]; out[1] = L; }
      out[2 + d] = O;
    }
  }
  // Private workspace: the partials are written; the grid completes only after the previous
  // kernel in the stream has.
  if (P.spec && P.ws_private) asm volatile("griddepcontrol.wait;\n" ::: "memory");
}

// Merge the per-CTA partials of one query head -- from the CTAs whose unit ranges cover its
// (KV head, query chunk) -- with the partial of the tokens after the pages, and write the
// output.  One CTA per query head; two threads per channel in the merge.  Launched as a
// programmatic dependent of the page pass: its CTAs become resident while that grid runs (they
// share the SM with a page-pass CTA) and compute the dense-tail partial then;
// griddepcontrol.wait releases them once the page pass has completed and its memory is
// visible, so no fence or atomic sits on the merge path.  The records' offsets are computed
// before the wait; after it they are staged in shared memory by concurrent 16-byte cp.async
// copies (one memory round trip per 64 records).
//
// Fused decode step (P.fused): the kernel also appends the new token of every KV head, as
// TurboPolarKVCacheRuntime.append does before attention (turbo_polar_cache.py:106-161).
// Without a flush, the new token joins the dense-tail partial straight from k_new/v_new and
// one CTA per KV head stores it in the tail.  When it completes the tail's page, every CTA of
// that KV head encodes the page in shared memory (bit-exact codec, the same for all of them),
// one stores it as pool page n_pages, and each computes its query head's partial over the
// page's decoded keys and values.  The state words advance after the merge, written by the
// last CTA to have read them (a ticket in d_state[5]), so no CTA of this launch can see the
// new state.
constexpr int kCombineThreads = 256;
constexpr int kCombineWarps = kCombineThreads / 32;
constexpr int kCombineChunk = 64;

__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}

template <typename T>
__device__ __forceinline__ float4 load4(const T* p) {
  if (sizeof(T) == 4) return *reinterpret_cast<const float4*>(p);
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(u32_as_h2(u.x)), b = __half22float2(u32_as_h2(u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// Query head qh as the kernels read it: float16 (a float32 query is rounded), channels
// 4*lane .. 4*lane+3.
__device__ __forceinline__ float4 load_q4(const AttnParams& P, int qh, int lane) {
  const int64_t qi = int64_t(qh) * kD + 4 * lane;
  if (!P.q_f32) return load4(static_cast<const __half*>(P.q) + qi);
  float4 q4 = load4(static_cast<const float*>(P.q) + qi);
  q4.x = __half2float(__float2half_rn(q4.x)); q4.y = __half2float(__float2half_rn(q4.y));
  q4.z = __half2float(__float2half_rn(q4.z)); q4.w = __half2float(__float2half_rn(q4.w));
  return q4;
}

// Softmax partial of one query head over at most 64 tokens whose keys and values `kv(t, lane,
// k, v)` produces (channels 4*lane .. 4*lane+3 of token t).  Warp w owns tokens w, w+8, ...,
// w+56; every key of a warp is fetched before any is used.  Returns (m, l, o[channel tid]) in
// the base-2 domain for tid < 128.  metal.py:305-321 treats these tokens as plain keys and
// values.
template <class KV>
__device__ __forceinline__ void block_partial(const AttnParams& P, int qh, int valid, KV kv, float* s_sc, float* s_o,
                                              float& m_out, float& l_out, float& o_out) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int kPer = kPage / kCombineWarps;
  const float4 q4 = load_q4(P, qh, lane);
  float4 x[kPer];  // keys, then values
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int t = warp + kCombineWarps * j;
    x[j] = t < valid ? kv(t, lane, true) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    float dot = q4.x * x[j].x + q4.y * x[j].y + q4.z * x[j].z + q4.w * x[j].w;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    const int t = warp + kCombineWarps * j;
    if (lane == 0 && t < valid) s_sc[t] = dot * P.scale_log2;
  }
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int t = warp + kCombineWarps * j;
    x[j] = t < valid ? kv(t, lane, false) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  float m = -INFINITY;
  for (int t = 0; t < valid; ++t) m = fmaxf(m, s_sc[t]);
  float l = 0.f;
  float4 o4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int t = warp + kCombineWarps * j;
    if (t < valid) {
      const float p = exp2_approx(s_sc[t] - m);
      l += p;
      o4.x = fmaf(p, x[j].x, o4.x); o4.y = fmaf(p, x[j].y, o4.y);
      o4.z = fmaf(p, x[j].z, o4.z); o4.w = fmaf(p, x[j].w, o4.w);
    }
  }
  reinterpret_cast<float4*>(s_o + warp * kD)[lane] = o4;
  if (lane == 0) s_sc[kPage + warp] = l;
  __syncthreads();
  if (tid < kD) {
    float o = 0.f;
    l = 0.f;
#pragma unroll
    for (int w = 0; w < kCombineWarps; ++w) {
      o += s_o[w * kD + tid];
      l += s_sc[kPage + w];
    }
    m_out = m;
    l_out = l;
    o_out = o;
  }
  __syncthreads();
}

// One page of one KV head held in shared memory, laid out as a pool page block (the fused
// step's flush).
struct SmemPage {
  uint8_t codes[kPage * kPairs];  // encode scratch: one code per pair
  float red[8];                   // encode scratch: block reduction
  __align__(16) uint8_t block[kMaxPageBytes];
  float2 cs[2 * kLutEntries];     // float32 (cos, sin) per code: level-1 [0, 256), deep [256, 512)
  __half radii_scale;
};

union CombineSmem {
  float recs[kCombineChunk][kRecFloats];
  SmemPage page;
};

// Key and value channels 4*lane .. 4*lane+3 of token t of the shared-memory page, decoded as
// rfsn_v11/quant/polar/decoder.py:36-67 and v_quant/encoder.py:32-38 do (cos and sin of the
// code angle from the float16 table the page pass uses).
__device__ __forceinline__ float4 page_token(const AttnParams& P, SmemPage& pg, int t, int lane, bool key) {
  const PoolArgs& W = P.wpool;
  if (!key) {
    float vx[4];
    const float s = __half2float(*vscale_at(W, pg.block, t, lane >> 3));
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int8_t code = int8_t(*vcode_at(W, pg.block, t, 4 * lane + e) ^ 0x80u);
      vx[e] = __half2float(__float2half_rn(float(code) * s));
    }
    return make_float4(vx[0], vx[1], vx[2], vx[3]);
  }
  float kx[4];
  const float2* lut = pg.cs;
  const uint8_t* row = codes_at(W, pg.block, t);
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int j = 2 * lane + e;
    uint32_t code;
    float2 c2;
    if (j < P.l1_pairs) {
      code = P.l1_bits == 8 ? row[j] : (row[j >> 1] >> (4 * (j & 1))) & 15u;
      c2 = lut[code];
    } else {
      const uint8_t* drow = row + P.l1_row;
      const int rel = j - P.l1_pairs;
      if (P.deep_bits == 8) code = drow[rel];
      else if (P.deep_bits == 4) code = (drow[rel >> 1] >> (4 * (rel & 1))) & 15u;
      else code = (drow[rel >> 2] >> (2 * (rel & 3))) & 3u;
      c2 = lut[kLutEntries + code];
    }
    float r;
    if (P.int8_radii) {
      const float arg = __fmul_rn(float(*radius_i8_at(W, pg.block, t, j)), __half2float(pg.radii_scale));
      r = d2f(exp(double(arg)));
    } else {
      r = __half2float(*radius_f16_at(W, pg.block, t, j));
    }
    kx[2 * e] = __half2float(__float2half_rn(__fmul_rn(r, c2.x)));
    kx[2 * e + 1] = __half2float(__float2half_rn(__fmul_rn(r, c2.y)));
  }
  return make_float4(kx[0], kx[1], kx[2], kx[3]);
}

template <typename T>
__device__ __forceinline__ void dense_tail_partial(const AttnParams& P, int kvh, int qh, int valid, int new_at,
                                                   float* s_sc, float* s_o, float& M, float& L, float& O) {
  const T* tk = static_cast<const T*>(P.tail_k) + int64_t(kvh) * kPage * kD;
  const T* tv = static_cast<const T*>(P.tail_v) + int64_t(kvh) * kPage * kD;
  const T* nk = static_cast<const T*>(P.k_new) + int64_t(kvh) * P.new_head_stride;
  const T* nv = static_cast<const T*>(P.v_new) + int64_t(kvh) * P.new_head_stride;
  block_partial(P, qh, valid, [&](int t, int lane, bool key) {
    const bool nw = t == new_at;
    return key ? load4((nw ? nk : tk + t * kD) + 4 * lane) : load4((nw ? nv : tv + t * kD) + 4 * lane);
  }, s_sc, s_o, M, L, O);
}

// Kept out of line: the page encode needs more registers than the merge path may use.
template <typename T>
__device__ __noinline__ float3 flush_partial(const AttnParams& P, CombineSmem& sm, int kvh, int qh, int page,
                                              bool store, int valid, float* s_sc, float* s_o) {
  SmemPage& pg = sm.page;
  const T* tk = static_cast<const T*>(P.tail_k) + int64_t(kvh) * kPage * kD;
  const T* tv = static_cast<const T*>(P.tail_v) + int64_t(kvh) * kPage * kD;
  // Decoder tables for page_token (the encode's closing barrier orders them before the reads).
  for (int i = threadIdx.x; i < 2 * kLutEntries; i += blockDim.x) {
    const int bits = i < kLutEntries ? P.l1_bits : P.deep_bits, code = i & (kLutEntries - 1);
    pg.cs[i] = code < (1 << bits) ? cos_sin_of_code(code, bits) : make_float2(0.f, 0.f);
  }
  encode_page<T>(tk, tv, kD, P.wpool, pg.block, &pg.radii_scale, pg.codes, pg.red,
                 static_cast<const T*>(P.k_new) + int64_t(kvh) * P.new_head_stride,
                 static_cast<const T*>(P.v_new) + int64_t(kvh) * P.new_head_stride);
  if (store) store_page_block(P.wpool, pg.block, pg.radii_scale, kvh, page);
  float M = -INFINITY, L = 0.f, O = 0.f;
  block_partial(P, qh, valid, [&](int t, int lane, bool key) { return page_token(P, pg, t, lane, key); }, s_sc, s_o,
                M, L, O);
  return make_float3(M, L, O);
}

// ----------------------------------------------------------------------------- cross-GPU exchange
// Exchange buffer of one rank: records [2][world][H_q][kExchWords] of 64-bit words written by
// every rank into every rank's buffer (peer stores over NVLink), then this rank's epoch word and
// ticket.  A word holds one float of a record (m, l, o[128]) in its low half and the call's
// epoch in its high half, so a reader knows a word is current from the word alone: an
// aligned 64-bit store is single-copy atomic, and no fence or flag is needed between the
// data and its validity (one one-way NVLink trip instead of store, release fence, flag store).
//
// The records of epoch e go to slot e & 1.  With one slot, a rank that finished reading epoch e
// could publish e + 1 over its epoch-e record in a slower rank's buffer before that rank had
// read it, and the slower rank would wait until its budget ran out.  With two, a rank writes
// slot e & 1 again only at epoch e + 2, after it has read every rank's epoch e + 1 record; a
// rank publishes e + 1 only after its epoch-e merge has completed (consecutive calls on one
// exchange never overlap: the split combine of e + 1 starts its exchange after the page pass of
// e + 1 has completed, which waited for the split combine of e to complete), so by then every
// rank has finished reading slot e & 1.
constexpr int kExchWords = TP_PARTIAL_FLOATS;
__host__ __device__ inline size_t x_epoch_off(int world, int hq) {
  return (2 * size_t(world) * hq * kExchWords * sizeof(uint64_t) + 255) & ~size_t(255);
}

__device__ __forceinline__ void st_word_sys(uint64_t* p, float v, uint32_t epoch) {
  const uint64_t w = uint64_t(__float_as_uint(v)) | (uint64_t(epoch) << 32);
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;\n" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ld_word_sys(const uint64_t* p) {
  uint64_t w;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];\n" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// Publish this rank's merged (m, l, o) of query head qh to every rank, wait (bounded) until
// every rank's record of qh for this epoch is here, and merge them.  Threads d < 128 hold
// channel d.  False after a wait ran out (a rank that never published).
__device__ __forceinline__ bool exchange_merge(const AttnParams& P, int qh, int epoch, float& M, float& L, float& O) {
  const int tid = threadIdx.x;
  const int W = P.xworld, hq = P.num_q_heads;
  const uint32_t ep = uint32_t(epoch);
  const size_t slot = size_t(ep & 1u) * W;  // first record of this epoch's slot, in records of H_q
  if (tid < kD) {
    for (int r = 0; r < W; ++r) {
      uint64_t* rec = reinterpret_cast<uint64_t*>(P.xbuf[r]) + ((slot + P.xrank) * hq + qh) * kExchWords;
      st_word_sys(rec + 2 + tid, O, ep);
      if (tid == 0) {
        st_word_sys(rec, M, ep);
        st_word_sys(rec + 1, L, ep);
      }
    }
  }
  __shared__ int s_ok;
  __shared__ float s_x[3][kD];
  if (tid == 0) s_ok = 1;
  __syncthreads();
  // Threads t and t + 128 take channel t & 127, the first the even ranks and the second the odd
  // ones.  A pass loads the (m, l, o[channel]) words of two ranks still missing before it checks
  // either, so once the records are here the wait costs one memory round trip for up to 4 ranks
  // and two for 8, not one per rank.
  constexpr int kPer = TP_MAX_RANKS / 2;
  const int d = tid & (kD - 1), par = tid >> 7;
  const uint64_t* base = reinterpret_cast<const uint64_t*>(P.xbuf[P.xrank]) + (slot * hq + qh) * kExchWords;
  float m[kPer], l[kPer], o[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    m[j] = -INFINITY;
    l[j] = o[j] = 0.f;
  }
  bool ok = true;
  const long long t0 = clock64();
#pragma unroll
  for (int jg = 0; jg < kPer; jg += 2) {
    bool got0 = 2 * jg + par >= W, got1 = 2 * (jg + 1) + par >= W;  // ranks beyond the world: nothing
    while (ok && !(got0 && got1)) {
      uint64_t w0[3], w1[3];
      if (!got0) {
        const uint64_t* rec = base + size_t(2 * jg + par) * hq * kExchWords;
        w0[0] = ld_word_sys(rec);
        w0[1] = ld_word_sys(rec + 1);
        w0[2] = ld_word_sys(rec + 2 + d);
      }
      if (!got1) {
        const uint64_t* rec = base + size_t(2 * (jg + 1) + par) * hq * kExchWords;
        w1[0] = ld_word_sys(rec);
        w1[1] = ld_word_sys(rec + 1);
        w1[2] = ld_word_sys(rec + 2 + d);
      }
      if (!got0 && uint32_t(w0[0] >> 32) == ep && uint32_t(w0[1] >> 32) == ep && uint32_t(w0[2] >> 32) == ep) {
        got0 = true;
        m[jg] = __uint_as_float(uint32_t(w0[0]));
        l[jg] = __uint_as_float(uint32_t(w0[1]));
        o[jg] = __uint_as_float(uint32_t(w0[2]));
      }
      if (!got1 && uint32_t(w1[0] >> 32) == ep && uint32_t(w1[1] >> 32) == ep && uint32_t(w1[2] >> 32) == ep) {
        got1 = true;
        m[jg + 1] = __uint_as_float(uint32_t(w1[0]));
        l[jg + 1] = __uint_as_float(uint32_t(w1[1]));
        o[jg + 1] = __uint_as_float(uint32_t(w1[2]));
      }
      if (clock64() - t0 > (1ll << 31)) ok = false;
    }
  }
  if (!ok) s_ok = 0;
  float Mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kPer; ++j) Mx = fmaxf(Mx, m[j]);
  float Lx = 0.f, Ox = 0.f;
  if (Mx != -INFINITY) {
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const float w = (m[j] == -INFINITY) ? 0.f : exp2_approx(m[j] - Mx);
      Lx = fmaf(l[j], w, Lx);
      Ox = fmaf(o[j], w, Ox);
    }
  }
  if (par) {
    s_x[0][d] = Mx;
    s_x[1][d] = Lx;
    s_x[2][d] = Ox;
  }
  __syncthreads();
  if (!par) {
    const float m1 = s_x[0][d], l1 = s_x[1][d], o1 = s_x[2][d];
    const float Mt = fmaxf(Mx, m1);
    float Lt = 0.f, Ot = 0.f;
    if (s_ok && Mt != -INFINITY) {
      const float a0 = (Mx == -INFINITY) ? 0.f : exp2_approx(Mx - Mt);
      const float a1 = (m1 == -INFINITY) ? 0.f : exp2_approx(m1 - Mt);
      Lt = Lx * a0 + l1 * a1;
      Ot = Ox * a0 + o1 * a1;
    }
    M = Mt;
    L = Lt;
    O = Ot;
  }
  __syncthreads();
  return s_ok != 0;
}

// Fused step: advance the state words once every CTA has read them (ticket) and the page pass
// has completed (griddepcontrol.wait), then reset the ticket.
__device__ __forceinline__ void advance_state(const AttnParams& P, const tp_state& st, int n_pages, int tail_len,
                                              bool appended, bool flush) {
  if (appended) {
    P.d_state[0] = n_pages + (flush ? 1 : 0);
    P.d_state[1] = flush ? 0 : tail_len + 1;
    P.d_state[2] = st.seq_len + 1;
  }
  P.d_state[5] = 0;
}

// At most 48 registers a thread (five CTAs on an SM once the page pass has finished; one fits
// beside a page-pass CTA of up to 192 registers).
__global__ void __launch_bounds__(kCombineThreads, 5) split_combine_kernel(const __grid_constant__ AttnParams P) {
  __shared__ __align__(16) CombineSmem sm;
  __shared__ int soff[kMaxContrib];
  __shared__ __align__(16) float s_o[kCombineWarps * kD];
  __shared__ float s_sc[kPage + kCombineWarps];
  __shared__ int s_last, s_epoch;
  const int tid = threadIdx.x;
  const int vh = blockIdx.x / P.gmax, h = blockIdx.x % P.gmax;
  const int kvh = vh / P.nqc, chunk = vh % P.nqc;
  const int gc = min(kMaxHeads, P.group - chunk * kMaxHeads);
  // The next page pass in the stream may start now: it waits for this grid to complete before
  // it reads anything this call writes (or, when it shares no buffer with this call, before it
  // writes its partials).
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

  // One thread reads the state words; with the fused step it then takes a ticket, and the
  // CTA holding the last ticket advances the words after the merge.
  __shared__ tp_state s_st;
  if (tid == 0) {
    tp_state st = P.st;
    if (P.d_state) {
      st.n_pages = P.d_state[0];
      st.tail_len = P.d_state[1];
      st.seq_len = P.d_state[2];
      st.first_page = P.d_state[3];
    }
    s_st = st;
    s_last = 0;
    if (P.xworld > 1) {
      // Exchange epoch: read by every CTA, advanced by the last to have read it.
      int* ew = reinterpret_cast<int*>(P.xbuf[P.xrank] + x_epoch_off(P.xworld, P.num_q_heads));
      const int e = ew[0] + 1;
      s_epoch = e;
      __threadfence();
      if (atomicAdd(&ew[1], 1) == int(gridDim.x) - 1) {
        ew[0] = e;
        ew[1] = 0;
      }
    }
    if (P.fused) {
      __threadfence();  // the reads above happen before the ticket
      s_last = atomicAdd(&P.d_state[5], 1) == int(gridDim.x) - 1;
    }
  }
  __syncthreads();
  const tp_state st = s_st;
  const int n_pages = min(max(st.n_pages, 0), P.page_capacity);
  const int tail_len = min(max(st.tail_len, 0), kPage);
  const int64_t tpos0 = (int64_t(st.first_page) + n_pages) * kPage;
  // Fused step: the new token goes to tail index tail_len; it completes a page when that is 63.
  const bool flush = P.fused && tail_len == kPage - 1;
  const bool appended = P.fused && tail_len < kPage && !(flush && n_pages >= P.page_capacity);
  if (h >= gc) {
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    if (s_last && tid == 0) advance_state(P, st, n_pages, tail_len, appended, flush);
    return;
  }
  const int qh = kvh * P.group + chunk * kMaxHeads + h;
  const bool designated = chunk == 0 && h == 0;
  float M = -INFINITY, L = 0.f, O = 0.f;
  if (appended && flush) {
    const int valid = int(clamp64(int64_t(st.seq_len) + 1 - tpos0, 0, kPage));
    const float3 r = P.tail_f32 ? flush_partial<float>(P, sm, kvh, qh, n_pages, designated, valid, s_sc, s_o)
                                : flush_partial<__half>(P, sm, kvh, qh, n_pages, designated, valid, s_sc, s_o);
    M = r.x;
    L = r.y;
    O = r.z;
  } else {
    const int len = tail_len + (appended ? 1 : 0);
    const int valid = int(clamp64(int64_t(st.seq_len) + (appended ? 1 : 0) - tpos0, 0, len));
    const int new_at = appended ? tail_len : -1;
    if (valid > 0) {
      if (P.tail_f32) dense_tail_partial<float>(P, kvh, qh, valid, new_at, s_sc, s_o, M, L, O);
      else dense_tail_partial<__half>(P, kvh, qh, valid, new_at, s_sc, s_o, M, L, O);
    }
    if (appended && designated) {
      const int esz = P.tail_f32 ? 4 : 2;
      const uint8_t* nk = static_cast<const uint8_t*>(P.k_new) + int64_t(kvh) * P.new_head_stride * esz;
      const uint8_t* nv = static_cast<const uint8_t*>(P.v_new) + int64_t(kvh) * P.new_head_stride * esz;
      uint8_t* tk = static_cast<uint8_t*>(P.tail_k) + (int64_t(kvh) * kPage + tail_len) * kD * esz;
      uint8_t* tv = static_cast<uint8_t*>(P.tail_v) + (int64_t(kvh) * kPage + tail_len) * kD * esz;
      for (int i = tid; i < kD * esz / 4; i += kCombineThreads) {
        reinterpret_cast<uint32_t*>(tk)[i] = reinterpret_cast<const uint32_t*>(nk)[i];
        reinterpret_cast<uint32_t*>(tv)[i] = reinterpret_cast<const uint32_t*>(nv)[i];
      }
    }
  }
  // Token dropped: 1 = tail state out of range, 2 = page pool full.
  if (P.fused && !appended && tid == 0 && designated) P.d_state[4] = tail_len >= kPage ? 1 : 2;

  // The page pass's partition, recomputed from the same state it read, and the workspace
  // offset of every record to merge: all known before the page pass completes.
  const Grid g = grid_of(P.num_kv_heads * P.nqc, n_pages, P.main_grid);
  int n = 0;
  if (P.owner) {
    n = n_pages > 0 ? kConsumers : 0;  // the owning CTA's warps' records of this segment
    if (tid < n) soff[tid] = (vh * kConsumers + tid) * kPartialStride + h * kRecFloats;
  } else if (g.U > 0) {
    const int c_lo = part_owner(g, vh * g.uph);
    n = part_owner(g, vh * g.uph + g.uph - 1) - c_lo + 1;
    for (int ci = tid; ci < n; ci += kCombineThreads) {
      const int cc = c_lo + ci;
      soff[ci] = (cc * 2 + (vh - part_begin(g, cc) / g.uph)) * kPartialStride + h * kRecFloats;
    }
  }
  __syncthreads();

  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  // Two threads per channel: thread t adds weight x o over the records of parity t >> 7 for
  // channel t & 127 (the dense-tail partial starts in half 0).  Warp 0 takes each chunk's new
  // maximum, the factor that rescales what was merged before, every record's weight
  // exp2(m - max) and the new sum, once for all channels.
  const int d = tid & (kD - 1), half = tid >> 7;
  __shared__ float s_w[kCombineChunk], s_run[3];  // weights; running max, sum, rescale factor
  static_assert(kCombineChunk == 64, "warp 0 takes two records a lane");
  float Oh = half ? 0.f : O;
  if (tid == 0) {
    s_run[0] = M;
    s_run[1] = L;
  }
#pragma unroll 1
  for (int c0 = 0; c0 < n; c0 += kCombineChunk) {
    const int cn = min(kCombineChunk, n - c0);
    constexpr int kQuads = kRecFloats / 4;
    for (int i = tid; i < cn * kQuads; i += kCombineThreads) {
      const int ci = i / kQuads, e = 4 * (i - ci * kQuads);
      cp_async16(&sm.recs[ci][e], P.ws_partials + soff[c0 + ci] + e);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    if (tid < 32) {
      const float M0 = s_run[0];
      const bool has0 = tid < cn, has1 = tid + 32 < cn;
      const float m0 = has0 ? sm.recs[tid][0] : -INFINITY, m1 = has1 ? sm.recs[tid + 32][0] : -INFINITY;
      float Mc = fmaxf(M0, fmaxf(m0, m1));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) Mc = fmaxf(Mc, __shfl_xor_sync(0xffffffffu, Mc, o));
      const float a = (M0 == -INFINITY) ? 0.f : exp2_approx(M0 - Mc);
      const float w0 = (m0 == -INFINITY) ? 0.f : exp2_approx(m0 - Mc);
      const float w1 = (m1 == -INFINITY) ? 0.f : exp2_approx(m1 - Mc);
      if (has0) s_w[tid] = w0;
      if (has1) s_w[tid + 32] = w1;
      float l = (has0 ? sm.recs[tid][1] * w0 : 0.f) + (has1 ? sm.recs[tid + 32][1] * w1 : 0.f);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      if (tid == 0) {
        s_run[1] = fmaf(s_run[1], a, l);
        s_run[0] = Mc;
        s_run[2] = a;
      }
    }
    __syncthreads();
    Oh *= s_run[2];
#pragma unroll 4
    for (int ci = half; ci < cn; ci += 2) Oh = fmaf(sm.recs[ci][2 + d], s_w[ci], Oh);
    __syncthreads();
  }
  if (half) s_o[d] = Oh;
  __syncthreads();
  if (!half) {
    O = Oh + s_o[d];
    M = s_run[0];
    L = s_run[1];
  }
  __syncthreads();
  if (P.xworld > 1) {
    if (!exchange_merge(P, qh, s_epoch, M, L, O) && tid == 0) atomicExch(P.ws_error, 3);  // a rank missing
  }
  if (tid < kD) write_result(P, qh, tid, M, L, O);
  if (s_last && tid == 0) advance_state(P, st, n_pages, tail_len, appended, flush);
}

// Plain attention (no decode step, no exchange) over more (KV head, query chunk) segments than
// SMs, as a batch of sequences gives: one CTA per segment merges all gc query heads of the
// segment, instead of one CTA per query head.  A workspace record holds the partials of every
// head of its segment side by side, so one round of copies stages the records of all heads;
// the heads' dense-tail partials run one after another before griddepcontrol.wait.  Per chunk
// of records, thread h of the CTA takes head h's new maximum, the factor that rescales what
// was merged before, the weight exp2(m - max) of every record and the new sum, once for all
// 128 channels; each channel thread then rescales its accumulators and adds weight x o per
// record (recomputing the weights in every channel thread, as split_combine_kernel does for
// its one head, made this kernel instruction-bound at about 1,050 instructions a thread).  A
// segment has at most 7 records here (whole-segment partition: one per compute warp; whole
// waves: at most three CTAs), so one chunk holds them all.  Launched as a programmatic dependent of the
// page pass like split_combine_kernel; its static shared memory is no larger, so a CTA fits
// beside a page-pass CTA.
constexpr int kSegRecs = 56;  // records of the staging area in one chunk (the rest: tail partials)
__global__ void __launch_bounds__(kCombineThreads, 4) segment_combine_kernel(const __grid_constant__ AttnParams P) {
  __shared__ __align__(16) float recs[kCombineChunk * kRecFloats];
  __shared__ int soff[kMaxContrib];
  __shared__ __align__(16) float s_o[kCombineWarps * kD];
  __shared__ float s_sc[kPage + kCombineWarps];
  __shared__ float s_tm[kMaxHeads][2];
  __shared__ tp_state s_st;
  float* s_to = recs + kSegRecs * kRecFloats;  // tail partials o[h][128], until the records land
  static_assert((kCombineChunk - kSegRecs) * kRecFloats >= kMaxHeads * kD, "tail partials");
  const int tid = threadIdx.x;
  const int vh = blockIdx.x;
  const int kvh = vh / P.nqc, chunk = vh % P.nqc;
  const int gc = min(kMaxHeads, P.group - chunk * kMaxHeads);
  const int qh0 = kvh * P.group + chunk * kMaxHeads;
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  if (tid == 0) s_st = read_state(P);
  __syncthreads();
  const tp_state st = s_st;
  const int n_pages = min(max(st.n_pages, 0), P.page_capacity);
  const int tail_len = min(max(st.tail_len, 0), kPage);
  const int64_t tpos0 = (int64_t(st.first_page) + n_pages) * kPage;
  const int valid = int(clamp64(int64_t(st.seq_len) - tpos0, 0, tail_len));
  const int d = tid & (kD - 1), half = tid >> 7;
  for (int h = 0; h < gc; ++h) {
    float M = -INFINITY, L = 0.f, O = 0.f;
    if (valid > 0) {
      if (P.tail_f32) dense_tail_partial<float>(P, kvh, qh0 + h, valid, -1, s_sc, s_o, M, L, O);
      else dense_tail_partial<__half>(P, kvh, qh0 + h, valid, -1, s_sc, s_o, M, L, O);
    }
    if (tid < kD) {
      s_to[h * kD + tid] = O;
      if (tid == 0) { s_tm[h][0] = M; s_tm[h][1] = L; }
    }
  }
  // Record offsets (of the segment's first head), as split_combine_kernel computes them.
  const Grid g = grid_of(P.num_kv_heads * P.nqc, n_pages, P.main_grid);
  int n = 0;
  if (P.owner) {
    n = n_pages > 0 ? kConsumers : 0;
    if (tid < n) soff[tid] = (vh * kConsumers + tid) * kPartialStride;
  } else if (g.U > 0) {
    const int c_lo = part_owner(g, vh * g.uph);
    n = part_owner(g, vh * g.uph + g.uph - 1) - c_lo + 1;
    for (int ci = tid; ci < n; ci += kCombineThreads) {
      const int cc = c_lo + ci;
      soff[ci] = (cc * 2 + (vh - part_begin(g, cc) / g.uph)) * kPartialStride;
    }
  }
  __syncthreads();
  // Thread (half, d) owns channel d of heads half, half + 2, ...; the per-head running maximum,
  // sum and rescale factor and the per-(record, head) weights are computed once, by thread h
  // for head h, and read by every channel.
  __shared__ float s_M[kMaxHeads], s_L[kMaxHeads], s_a[kMaxHeads], s_w[kSegRecs];
  constexpr int kOwn = kMaxHeads / 2;
  float Oh[kOwn];
#pragma unroll
  for (int j = 0; j < kOwn; ++j) {
    const int h = half + 2 * j;
    Oh[j] = h < gc ? s_to[h * kD + d] : 0.f;
  }
  if (tid < gc) {
    s_M[tid] = s_tm[tid][0];
    s_L[tid] = s_tm[tid][1];
  }
  const int rc = kSegRecs / gc;  // records per chunk, all heads of each
  const int rfl = gc * kRecFloats;
  const int q4 = rfl / 4;
  __syncthreads();  // the tail partials are read before the records overwrite the staging area

  asm volatile("griddepcontrol.wait;\n" ::: "memory");
#pragma unroll 1
  for (int c0 = 0; c0 < n; c0 += rc) {
    const int cn = min(rc, n - c0);
    for (int ci = 0; ci < cn; ++ci) {
      const float* src = P.ws_partials + soff[c0 + ci];
      for (int e = tid; e < q4; e += kCombineThreads) cp_async16(&recs[ci * rfl + 4 * e], src + 4 * e);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    if (tid < gc) {
      const int h = tid;
      const float* r = recs + h * kRecFloats;
      const float M0 = s_M[h];
      float Mc = M0;
      for (int ci = 0; ci < cn; ++ci) Mc = fmaxf(Mc, r[ci * rfl]);
      const float a = (M0 == -INFINITY) ? 0.f : exp2_approx(M0 - Mc);
      float L = s_L[h] * a;
      for (int ci = 0; ci < cn; ++ci) {
        const float m = r[ci * rfl];
        const float w = (m == -INFINITY) ? 0.f : exp2_approx(m - Mc);
        s_w[ci * gc + h] = w;
        L = fmaf(r[ci * rfl + 1], w, L);
      }
      s_a[h] = a;
      s_M[h] = Mc;
      s_L[h] = L;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kOwn; ++j) {
      const int h = half + 2 * j;
      if (h >= gc) continue;
      const float* r = recs + h * kRecFloats + 2 + d;
      float O = Oh[j] * s_a[h];
      for (int ci = 0; ci < cn; ++ci) O = fmaf(r[ci * rfl], s_w[ci * gc + h], O);
      Oh[j] = O;
    }
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < kOwn; ++j) {
    const int h = half + 2 * j;
    if (h < gc) write_result(P, qh0 + h, d, s_M[h], s_L[h], Oh[j]);
  }
}

// ----------------------------------------------------------------------------- cross-shard combine
__global__ void combine_kernel(const float* partials, int n_parts, int num_q_heads, __half* out) {
  const int h = blockIdx.x, d = threadIdx.x;
  float M = -INFINITY;
  for (int r = 0; r < n_parts; ++r) M = fmaxf(M, partials[(int64_t(r) * num_q_heads + h) * TP_PARTIAL_FLOATS]);
  float L = 0.f, O = 0.f;
  if (M != -INFINITY) {
    for (int r = 0; r < n_parts; ++r) {
      const float* rec = partials + (int64_t(r) * num_q_heads + h) * TP_PARTIAL_FLOATS;
      if (rec[0] == -INFINITY) continue;
      const float f = exp2f(rec[0] - M);
      L += rec[1] * f;
      O += rec[2 + d] * f;
    }
  }
  out[int64_t(h) * kD + d] = __float2half_rn(L > 0.f ? O / L : 0.f);
}

// Launch configuration per device, worked out on the first call on that device and shared by
// every host thread (one mutex): the SM count, the shared memory the page pass may use and
// how much of it each page-pass variant has been allowed so far (cudaFuncSetAttribute acts on
// the current device).
constexpr int kModes = 3;
constexpr int kVariants = 4 * kModes;  // key format x (value codes, dense values) x partition
constexpr int kMaxDevices = 64;
struct DeviceCfg {
  int sms = 0;
  int ring_budget[kVariants][2] = {};  // [variant][room left for a split-combine CTA]
  int attr_bytes[kVariants] = {};
};
static std::mutex g_cfg_mutex;
static DeviceCfg g_cfg[kMaxDevices];

static DeviceCfg& device_cfg() {  // caller holds g_cfg_mutex
  int dev = 0;
  cudaGetDevice(&dev);
  return g_cfg[(dev >= 0 && dev < kMaxDevices) ? dev : 0];
}

static int num_sms() {
  std::lock_guard<std::mutex> lock(g_cfg_mutex);
  DeviceCfg& cfg = device_cfg();
  if (cfg.sms == 0) {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cfg.sms = n;
  }
  return cfg.sms;
}

// Dynamic shared memory the page pass (variant `variant`, kernel `page_pass`) may use: the opt-in
// per-block limit and, when the registers allow a split-combine CTA beside a page-pass CTA on
// one SM (so it starts, and finishes the dense tail, while the page pass runs), no more than
// leaves room for it (`leave_room`; the dense-value variants' stages are larger, and a long
// call takes the whole limit for two ring stages per compute warp instead of one).
static int ring_budget(int variant, const void* page_pass, bool leave_room) {
  std::lock_guard<std::mutex> lock(g_cfg_mutex);
  int& budget = device_cfg().ring_budget[variant][leave_room ? 1 : 0];
  if (budget == 0) {
    int dev = 0, per_sm = 233472, per_block = 232448, reserved = 1024, regs = 65536;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&per_block, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    cudaDeviceGetAttribute(&regs, cudaDevAttrMaxRegistersPerMultiprocessor, dev);
    cudaFuncAttributes comb = {}, pp = {};
    cudaFuncGetAttributes(&comb, reinterpret_cast<const void*>(split_combine_kernel));
    cudaFuncGetAttributes(&pp, page_pass);
    auto up8 = [](int r) { return (r + 7) / 8 * 8; };
    const bool beside = up8(pp.numRegs) * kThreads + up8(comb.numRegs) * kCombineThreads <= regs;
    budget = per_block - int(pp.sharedSizeBytes) - 256;
    if (beside && leave_room)
      budget = min(budget, per_sm - 2 * reserved - int(comb.sharedSizeBytes) - int(pp.sharedSizeBytes) - 256);
  }
  return budget;
}

// Let the page pass (variant `variant`) use `smem` bytes of dynamic shared memory on the current
// device, and all of the unified L1/shared array as shared memory for it and the split
// combine, so the split-combine CTAs fit beside a page-pass CTA.
static cudaError_t reserve_smem(int variant, const void* page_pass, int smem) {
  std::lock_guard<std::mutex> lock(g_cfg_mutex);
  int& have = device_cfg().attr_bytes[variant];
  if (smem <= have) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(page_pass, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(page_pass, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(reinterpret_cast<const void*>(split_combine_kernel),
                             cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(reinterpret_cast<const void*>(segment_combine_kernel),
                             cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e == cudaSuccess) have = smem;
  return e;
}

// (KV head, query chunk) segments of a head layout.
static int segments_of(int num_kv_heads, int num_q_heads) {
  const int group = num_q_heads / num_kv_heads;
  return num_kv_heads * ((group + kMaxHeads - 1) / kMaxHeads);
}

// Page-pass CTAs.  Up to one segment per SM: one CTA per SM (the flat partition).  With more
// segments than SMs (large batches), one wave of CTAs that each stream whole segments (the
// whole-segment partition, AttnParams::owner: the grid is then below the segment count) when
// the CTAs own nearly equal numbers of segments -- the largest share ceil(V / SMs) at most 1.25x
// the mean; otherwise whole waves of the flat partition, which stream equal numbers of units
// (each CTA between half a segment and one, a segment spread over at most three CTAs).
// Measured on B200 (8 KV heads per sequence, one call): 128 x 512 tokens 55 us whole-segment
// against 80 in waves, 64 x 1K 44 against 54, 40 x 4K 91 against 80, 19 x 4K 59 against 42.
static int grid_size(int num_kv_heads, int num_q_heads) {
  const int sms = num_sms(), segs = segments_of(num_kv_heads, num_q_heads);
  if (segs <= sms) return sms;
  const int waves = (segs + sms - 1) / sms;
  return 4 * waves * sms <= 5 * segs ? sms : waves * sms;
}

// Workspace record slots: two per CTA (flat partition), or one per segment and compute warp
// (whole-segment partition).
static int record_slots(int num_kv_heads, int num_q_heads) {
  const int grid = grid_size(num_kv_heads, num_q_heads), segs = segments_of(num_kv_heads, num_q_heads);
  return segs > grid ? segs * kConsumers : 2 * grid;
}

// float32 (cos, sin) of the decoder angle of a `bits`-bit code, on the host: the angle is
// evaluated as rfsn_v11/quant/polar/decoder.py:36-56 does (code / (2^bits - 1) * 2pi - pi, each op
// rounded to float32; evaluating in double and rounding gives the same floats), cos and sin in
// double rounded to float32 -- the values cos_sin_of_code gives on the device.
static float2 host_cos_sin(int code, int bits) {
  const int lm1 = (1 << bits) - 1;
  const float norm = float(double(code) / double(lm1));
  const float prod = float(double(norm) * double(6.28318530717958647692f));
  const float ang = float(double(prod) - double(3.14159265358979323846f));
  return make_float2(float(cos(double(ang))), float(sin(double(ang))));
}

// The launch's host-side decoder table for `mode` (AttnParams::cs).
static void fill_decoder_table(int mode, float2* cs) {
  for (int i = 0; i < kLutEntries; ++i) cs[i] = make_float2(0.f, 0.f);
  if (mode == kModeFast) {
    for (int c = 0; c < 16; ++c) {
      const float2 v = host_cos_sin(c, 4);
      const __half ch = __float2half_rn(v.x), sh = __float2half_rn(v.y);
      const __half cl = __float2half_rn(v.x - __half2float(ch)), sl = __float2half_rn(v.y - __half2float(sh));
      uint2 e;
      e.x = uint32_t(__half_as_ushort(ch)) | (uint32_t(__half_as_ushort(sh)) << 16);
      e.y = uint32_t(__half_as_ushort(cl)) | (uint32_t(__half_as_ushort(sl)) << 16);
      std::memcpy(&cs[c], &e, sizeof(e));
    }
  } else if (mode == kModeAdapter) {
    for (int c = 0; c < kLutEntries; ++c) cs[c] = host_cos_sin(c, 8);
  }
}

static StreamLog g_stream_log;  // last call's writes per stream (tp_overlap.h)

// The stream a launch on `s` goes to, as StreamLog tells streams apart: the current device, the
// handle, the host thread for the per-thread default stream, and the capture being recorded.
static StreamKey stream_key(cudaStream_t s) {
  StreamKey k{};
  cudaGetDevice(&k.device);
  k.stream = reinterpret_cast<uintptr_t>(s);
  if (s == cudaStreamPerThread) k.thread = uint64_t(std::hash<std::thread::id>{}(std::this_thread::get_id())) | 1u;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  unsigned long long id = 0;
  if (cudaStreamGetCaptureInfo(s, &cs, &id) != cudaSuccess) {
    cudaGetLastError();  // not capturing as far as the log is concerned; the launch reports errors
  } else if (cs == cudaStreamCaptureStatusActive) {
    k.capture = id ? id : 1;
  }
  return k;
}

// The page-pass kernels: one per key format, with value codes or dense values, flat or
// whole-segment partition.
template <int kMode, bool kDenseV, bool kOwner>
static cudaError_t launch_page_pass(const cudaLaunchConfig_t* c, const AttnParams& P) {
  return cudaLaunchKernelEx(c, decode_attention_kernel<kMode, kDenseV, kOwner>, P);
}
struct PagePass {
  const void* fn;
  cudaError_t (*launch)(const cudaLaunchConfig_t*, const AttnParams&);
};
template <int kMode, bool kDenseV, bool kOwner>
static PagePass page_pass_of() {
  return {reinterpret_cast<const void*>(decode_attention_kernel<kMode, kDenseV, kOwner>),
          launch_page_pass<kMode, kDenseV, kOwner>};
}
template <bool kDenseV, bool kOwner>
static PagePass page_pass_for(int mode) {
  return mode == kModeFast      ? page_pass_of<kModeFast, kDenseV, kOwner>()
         : mode == kModeAdapter ? page_pass_of<kModeAdapter, kDenseV, kOwner>()
                                : page_pass_of<kModeGeneral, kDenseV, kOwner>();
}
static PagePass page_pass(int mode, bool dense_v, bool owner) {
  if (dense_v) return owner ? page_pass_for<true, true>(mode) : page_pass_for<true, false>(mode);
  return owner ? page_pass_for<false, true>(mode) : page_pass_for<false, false>(mode);
}

// cuTensorMapEncodeTiled from the driver (resolved once; NULL when the driver lacks it).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

// Tensor map of a float16 value array [heads][tokens][128] (head_stride elements between heads):
// boxes of 64 channels x 32 tokens x 1 head, 128-byte swizzle, zero fill outside the array.
static int encode_value_map(CUtensorMap* m, const void* v, int64_t tokens, int heads, int64_t head_stride) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(TP_ERR_CUDA, "tp_decode_attention_dense_v: the driver has no cuTensorMapEncodeTiled");
  cuuint64_t dims[3] = {cuuint64_t(kD), cuuint64_t(tokens), cuuint64_t(heads)};
  cuuint64_t strides[2] = {cuuint64_t(kD * 2), cuuint64_t(head_stride * 2)};
  cuuint32_t box[3] = {64, cuuint32_t(kHalf), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(v), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TP_ERR_INVALID, "tp_decode_attention_dense_v: cannot describe the value array (CUresult " +
                                    std::to_string(int(r)) + ")");
  return TP_OK;
}

}  // namespace tp

using namespace tp;

extern "C" {

size_t tp_decode_attention_workspace_size(int32_t num_kv_heads, int32_t num_q_heads) {
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads) return 0;
  const size_t bytes = 256 + size_t(record_slots(num_kv_heads, num_q_heads)) * kPartialStride * sizeof(float);
  return (bytes + 255) & ~size_t(255);
}

// The new token of a fused decode step.
struct StepArgs {
  const void* k_new;
  const void* v_new;
  int64_t head_stride;
};

// The float16 value array of a dense-V call: [heads][tokens][128], heads head_stride elements apart.
struct DenseV {
  const void* v;
  int64_t head_stride;
  int64_t tokens;
};

static int run_attention(const tp_page_pool* pool, const tp_tail* tail, tp_state state, int32_t* d_state,
                         const void* q, int32_t q_dtype, int32_t num_q_heads, float scale, void* out,
                         float* partial_out, void* workspace, size_t workspace_bytes, void* stream,
                         const StepArgs* step, const tp_exchange* x = nullptr, const DenseV* dv = nullptr) {
  Layout L;
  int st = validate_pool(pool, &L);
  if (st != TP_OK) return st;
  const int hkv = pool->num_kv_heads;
  if (num_q_heads <= 0 || num_q_heads % hkv)
    return fail(TP_ERR_INVALID, "num_q_heads must be divisible by num_kv_heads for GQA");
  if (!q) return fail(TP_ERR_INVALID, "tp_decode_attention: q is NULL");
  if (q_dtype != TP_F16 && q_dtype != TP_F32) return fail(TP_ERR_INVALID, "q must be float16 or float32");
  if (!out && !partial_out) return fail(TP_ERR_INVALID, "tp_decode_attention: no output buffer");
  if (!(scale > 0.f)) return fail(TP_ERR_INVALID, "attention scale must be positive");
  if (!d_state) {
    if (state.n_pages < 0 || state.n_pages > pool->page_capacity)
      return fail(TP_ERR_INVALID, "n_pages outside the page pool");
    if (state.tail_len < 0 || state.tail_len > TP_PAGE_TOKENS) return fail(TP_ERR_INVALID, "tail_len must be in [0, 64]");
    if (state.n_pages == 0 && state.tail_len == 0) return fail(TP_ERR_INVALID, "attention over an empty cache");
  }
  if (!tail || ((d_state || state.tail_len > 0) && (!tail->k || !tail->v)))
    return fail(TP_ERR_INVALID, "tp_decode_attention: tail buffers missing");
  const size_t need = tp_decode_attention_workspace_size(hkv, num_q_heads);
  if (!workspace || workspace_bytes < need)
    return fail(TP_ERR_INVALID, "tp_decode_attention: workspace too small (need " + std::to_string(need) + " bytes)");
  if ((reinterpret_cast<uintptr_t>(q) & 15)) return fail(TP_ERR_INVALID, "q must be 16-byte aligned");

  AttnParams P;
  P.pages = static_cast<const uint8_t*>(pool->pages);
  P.radii_scales = static_cast<const __half*>(pool->radii_scales);
  P.page_capacity = pool->page_capacity;
  P.l1_bits = pool->fmt.l1_bits;
  P.deep_bits = pool->fmt.deep_bits;
  P.l1_pairs = L.l1_pairs;
  P.l1_row = L.l1_row;
  P.deep_row = L.deep_row;
  P.code_row = L.code_row;
  P.radii_row = L.radii_row;
  P.int8_radii = pool->fmt.int8_radii;
  P.unit_bytes = L.unit_bytes;
  P.tail_k = tail->k;
  P.tail_v = tail->v;
  P.tail_f32 = tail->dtype == TP_F32;
  P.st = state;
  P.d_state = d_state;
  P.q = q;
  P.q_f32 = q_dtype == TP_F32;
  P.num_q_heads = num_q_heads;
  P.num_kv_heads = hkv;
  P.group = num_q_heads / hkv;
  P.nqc = (P.group + kMaxHeads - 1) / kMaxHeads;
  P.gmax = P.group < kMaxHeads ? P.group : kMaxHeads;
  P.scale_log2 = scale * 1.4426950408889634f;
  P.out = static_cast<__half*>(out);
  P.partial_out = partial_out;
  const int grid = grid_size(hkv, num_q_heads);
  P.main_grid = grid;
  P.owner = hkv * P.nqc > grid ? 1 : 0;
  // CTAs sharing one segment: up to the grid with one wave of the flat partition, at most three
  // with more waves, one with the whole-segment partition.
  if (hkv * P.nqc <= num_sms() && grid > kMaxContrib)
    return fail(TP_ERR_UNSUPPORTED, "tp_decode_attention: more SMs than one head's partials can merge");
  P.ws_error = static_cast<int*>(workspace);  // word 0: error
  P.fused = step != nullptr;
  P.k_new = step ? step->k_new : nullptr;
  P.v_new = step ? step->v_new : nullptr;
  P.new_head_stride = step ? step->head_stride : 0;
  P.wpool = pool_args(*pool, L);
  P.xworld = 0;
  P.xrank = 0;
  for (int r = 0; r < TP_MAX_RANKS; ++r) P.xbuf[r] = nullptr;
  if (x) {
    if (x->world < 2 || x->world > TP_MAX_RANKS || x->rank < 0 || x->rank >= x->world)
      return fail(TP_ERR_INVALID, "exchange: world must be in [2, 8] and rank in [0, world)");
    if (!out || partial_out) return fail(TP_ERR_INVALID, "exchange: a sharded call writes `out` only");
    for (int r = 0; r < x->world; ++r) {
      if (!x->buffers[r] || (reinterpret_cast<uintptr_t>(x->buffers[r]) & 255))
        return fail(TP_ERR_INVALID, "exchange: every rank's buffer must be mapped and 256-byte aligned");
      P.xbuf[r] = static_cast<uint8_t*>(x->buffers[r]);
    }
    P.xworld = x->world;
    P.xrank = x->rank;
  }
  P.ws_partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + 256);
  // Half-page stage: one unit copied linearly (radii | v codes | angle codes | v scales), or
  // with dense values radii | angle codes | value rows (1024-byte aligned).
  auto up = [](int x, int a) { return (x + a - 1) / a * a; };
  P.off_vcodes = L.u_vcodes;
  P.off_codes = L.u_codes;
  P.off_vscales = L.u_vscales;
  P.stage_bytes = up(L.unit_bytes, 128);
  P.k_radii_bytes = L.u_vcodes;
  P.k_code_bytes = L.u_vscales - L.u_codes;
  P.k_src_codes = L.u_codes;
  P.off_vdense = 0;
  std::memset(&P.vmap, 0, sizeof(P.vmap));
  if (dv) {
    P.off_codes = P.k_radii_bytes;
    P.off_vdense = up(P.k_radii_bytes + P.k_code_bytes, 1024);
    P.stage_bytes = P.off_vdense + 2 * kHalf * 64 * 2;
    st = encode_value_map(&P.vmap, dv->v, dv->tokens, hkv, dv->head_stride);
    if (st != TP_OK) return st;
  }
  const int merge_bytes = kConsumers * P.gmax * TP_PARTIAL_FLOATS * int(sizeof(float));
  P.smem_bar_off = 0;                       // full and empty barrier per ring stage
  P.smem_lut_off = up(2 * kMaxStages * 8, 128);
  P.lut_deep = 1 << P.l1_bits;
  P.smem_merge_off = P.smem_lut_off + up(8 * ((1 << P.l1_bits) + (1 << P.deep_bits)), 128) + 256;
  P.smem_scale_off = up(P.smem_merge_off + merge_bytes, 128);
  P.smem_tab_off = P.smem_scale_off + up(kMaxStages * 4, 128);
  const int mode = (P.l1_bits == 4 && P.deep_bits == 4 && pool->fmt.split_dim == 64 && !P.int8_radii) ? kModeFast
                   : (P.int8_radii && pool->fmt.split_dim == 0 && P.deep_bits == 8)                 ? kModeAdapter
                                                                                                   : kModeGeneral;
  P.smem_qcc_off = up(P.smem_tab_off + (mode == kModeAdapter ? kLutEntries * 16 * 8 : 0), 128);
  P.smem_stage_off = up(P.smem_qcc_off + (TP_QK_CUDA_CORES ? kConsumers * kQccFloats * 4 : 0), 128);

  fill_decoder_table(mode, P.cs);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const PagePass pass = page_pass(mode, dv != nullptr, P.owner != 0);
  const void* fn = pass.fn;
  const int variant = mode + (dv ? kModes : 0) + (P.owner ? 2 * kModes : 0);
  // Ring stages: as many as fit while a split-combine CTA still fits beside the page-pass CTA
  // on one SM (so it starts, and finishes the dense tail, while the page pass runs); with dense
  // values 1024 bytes go to aligning the ring, and one stage per compute warp is accepted.  A
  // dense-value call whose compute warps have more than two units each takes the whole limit
  // instead (its stages are larger; measured on B200 at 32 query / 8 KV heads: 32K 23.7 us
  // against 28.1 with room for the split combine, 4K 8.6 against 6.1).
  const int align_slack = dv ? 1024 : 0;
  bool leave_room = true;
  if (dv) {
    const int64_t units = int64_t(hkv) * P.nqc * 2 * state.n_pages;
    leave_room = (units + int64_t(grid) * kConsumers - 1) / (int64_t(grid) * kConsumers) <= 2;
  }
  const int ring_bytes = ring_budget(variant, fn, leave_room) - P.smem_stage_off - align_slack;
  P.n_stages = min(kMaxStages, ring_bytes / P.stage_bytes) / kConsumers * kConsumers;
  if (P.n_stages < (dv ? 1 : 2) * kConsumers)
    return fail(TP_ERR_UNSUPPORTED, "tp_decode_attention: not enough shared memory for the page ring");
  const int smem = P.smem_stage_off + align_slack + P.n_stages * P.stage_bytes;
  {
    const cudaError_t e = reserve_smem(variant, fn, smem);
    if (e != cudaSuccess)
      return fail(TP_ERR_CUDA, std::string("tp_decode_attention: cannot reserve ") + std::to_string(smem) +
                                   " bytes of shared memory: " + cudaGetErrorString(e));
  }
  {
    CallBuffers b;
    const size_t pool_pages = size_t(hkv) * pool->page_capacity;
    b.q = q;
    b.q_bytes = size_t(num_q_heads) * kD * (P.q_f32 ? 4 : 2);
    b.pages = pool->pages;
    b.pages_bytes = pool_pages * L.page_bytes;
    b.radii_scales = pool->radii_scales;
    b.radii_scales_bytes = pool_pages * sizeof(__half);
    b.tail_k = tail->k;
    b.tail_v = tail->v;
    b.tail_bytes = size_t(hkv) * kPage * kD * (P.tail_f32 ? 4 : 2);
    b.d_state = d_state;
    b.state_bytes = TP_STATE_WORDS * sizeof(int32_t);
    // The kernels write partial_out when it is given, else out (write_result).
    b.out = partial_out ? static_cast<void*>(partial_out) : out;
    b.out_bytes = partial_out ? size_t(num_q_heads) * TP_PARTIAL_FLOATS * sizeof(float)
                              : size_t(num_q_heads) * kD * sizeof(__half);
    if (step) {
      b.step = true;
      b.k_new = step->k_new;
      b.v_new = step->v_new;
      b.new_bytes = (size_t(hkv - 1) * step->head_stride + kD) * (P.tail_f32 ? 4 : 2);
    }
    if (x) {
      b.exchange = P.xbuf[P.xrank];
      b.exchange_bytes = x_epoch_off(P.xworld, num_q_heads) + 256;
    }
    if (dv) {
      b.values = dv->v;
      b.values_bytes = size_t((hkv - 1) * dv->head_stride + dv->tokens * kD) * sizeof(__half);
    }
    Spans reads, writes, cache;
    call_spans(b, reads, writes);
    cache_spans(b, cache);
    bool cache_final = false;
    b.workspace = workspace;
    b.workspace_bytes = need;
    Spans ws;
    workspace_spans(b, ws);
    bool ws_clear = false;
    P.spec = g_stream_log.independent(stream_key(s), reads, writes, &cache, &cache_final, &ws, &ws_clear) ? 1 : 0;
    P.cache_final = cache_final ? 1 : 0;
    P.ws_private = ws_clear ? 1 : 0;
  }
  // The page pass is a programmatic dependent of whatever precedes it in the stream (a no-op
  // unless that kernel triggers early, as the split combine of a previous call does): its
  // CTAs load their code tables while that kernel finishes, or, when the previous call is
  // independent of this one, run the whole pass.
  {
    cudaLaunchConfig_t mc = {};
    mc.gridDim = dim3(grid);
    mc.blockDim = dim3(kThreads);
    mc.dynamicSmemBytes = smem;
    mc.stream = s;
    cudaLaunchAttribute ma[1];
    ma[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    ma[0].val.programmaticStreamSerializationAllowed = 1;
    mc.attrs = ma;
    mc.numAttrs = 1;
    const cudaError_t e = pass.launch(&mc, P);
    if (e != cudaSuccess) return fail(TP_ERR_CUDA, std::string("tp_decode_attention: ") + cudaGetErrorString(e));
  }
  // Split combine as a programmatic dependent launch of the attention grid: one CTA per query
  // head, or, for plain attention over more segments than SMs, one per segment.
  const bool per_segment = !P.fused && P.xworld <= 1 && hkv * P.nqc > num_sms();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(per_segment ? hkv * P.nqc : hkv * P.nqc * P.gmax);
  cfg.blockDim = dim3(kCombineThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, per_segment ? segment_combine_kernel : split_combine_kernel, P);
  if (e != cudaSuccess) return fail(TP_ERR_CUDA, std::string("tp_decode_attention (combine): ") + cudaGetErrorString(e));
  return TP_OK;
}

static int check_step_args(const tp_page_pool* pool, const tp_tail* tail, const int32_t* d_state, const void* k_new,
                           const void* v_new, int32_t kv_dtype, int64_t head_stride) {
  if (!d_state) return fail(TP_ERR_INVALID, "tp_decode_step: the state words are required");
  if (!pool || !tail) return fail(TP_ERR_INVALID, "tp_decode_step: NULL pool or tail");
  if (!k_new || !v_new) return fail(TP_ERR_INVALID, "tp_decode_step: NULL new token");
  if (kv_dtype != tail->dtype) return fail(TP_ERR_INVALID, "tp_decode_step: new token dtype must match the tail");
  if (kv_dtype != TP_F16 && kv_dtype != TP_F32) return fail(TP_ERR_INVALID, "only float16 and float32 inputs are supported");
  const int64_t esz = kv_dtype == TP_F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(k_new) & 15) || (reinterpret_cast<uintptr_t>(v_new) & 15) ||
      head_stride < kD || (head_stride * esz) % 16)
    return fail(TP_ERR_INVALID, "tp_decode_step: new token rows must be 16-byte aligned, heads >= 128 elements apart");
  return TP_OK;
}

int tp_decode_attention(const tp_page_pool* pool, const tp_tail* tail, tp_state state, const int32_t* d_state,
                        const void* q, int32_t q_dtype, int32_t num_q_heads, float scale, void* out,
                        float* partial_out, void* workspace, size_t workspace_bytes, void* stream) {
  // Without a step the kernels only read the state words.
  return run_attention(pool, tail, state, const_cast<int32_t*>(d_state), q, q_dtype, num_q_heads, scale, out,
                       partial_out, workspace, workspace_bytes, stream, nullptr);
}

int tp_decode_attention_dense_v(const tp_page_pool* pool, tp_state state, const void* v, int64_t v_head_stride,
                                int64_t v_tokens, const void* q, int32_t q_dtype, int32_t num_q_heads, float scale,
                                void* out, float* partial_out, void* workspace, size_t workspace_bytes,
                                void* stream) {
  if (!pool) return fail(TP_ERR_INVALID, "page pool is NULL");
  if (state.tail_len != 0 || state.first_page != 0)
    return fail(TP_ERR_INVALID, "tp_decode_attention_dense_v: pages only (tail_len and first_page must be 0)");
  if (state.n_pages < 1 || state.n_pages > pool->page_capacity)
    return fail(TP_ERR_INVALID, "tp_decode_attention_dense_v: n_pages must be in [1, page_capacity]");
  if (state.seq_len < 1 || int64_t(state.seq_len) > int64_t(state.n_pages) * TP_PAGE_TOKENS)
    return fail(TP_ERR_INVALID, "tp_decode_attention_dense_v: seq_len must be in [1, 64 * n_pages]");
  if (!v || (reinterpret_cast<uintptr_t>(v) & 15))
    return fail(TP_ERR_INVALID, "tp_decode_attention_dense_v: the value array must be 16-byte aligned");
  if (v_tokens < state.seq_len || v_tokens > (int64_t(1) << 31))
    return fail(TP_ERR_INVALID, "tp_decode_attention_dense_v: v_tokens must be in [seq_len, 2^31]");
  if (v_head_stride < v_tokens * kD || v_head_stride % 8 || v_head_stride >= (int64_t(1) << 39))
    return fail(TP_ERR_INVALID,
                "tp_decode_attention_dense_v: v_head_stride must be a multiple of 8, >= 128 * v_tokens and < 2^39");
  const tp_tail none = {nullptr, nullptr, TP_F16};
  const DenseV dv{v, v_head_stride, v_tokens};
  return run_attention(pool, &none, state, nullptr, q, q_dtype, num_q_heads, scale, out, partial_out, workspace,
                       workspace_bytes, stream, nullptr, nullptr, &dv);
}

int tp_decode_step(const tp_page_pool* pool, const tp_tail* tail, int32_t* d_state, const void* k_new,
                   const void* v_new, int32_t kv_dtype, int64_t head_stride, const void* q, int32_t q_dtype,
                   int32_t num_q_heads, float scale, void* out, float* partial_out, void* workspace,
                   size_t workspace_bytes, void* stream) {
  const int st = check_step_args(pool, tail, d_state, k_new, v_new, kv_dtype, head_stride);
  if (st != TP_OK) return st;
  StepArgs a{k_new, v_new, head_stride};
  tp_state none = {0, 0, 0, 0};
  return run_attention(pool, tail, none, d_state, q, q_dtype, num_q_heads, scale, out, partial_out, workspace,
                       workspace_bytes, stream, &a);
}

size_t tp_exchange_bytes(int32_t world, int32_t num_q_heads) {
  if (world < 2 || world > TP_MAX_RANKS || num_q_heads <= 0) return 0;
  return x_epoch_off(world, num_q_heads) + 256;
}

int tp_ipc_alloc(size_t bytes, void** ptr, void* handle_out) {
  if (!ptr || !handle_out || bytes == 0) return fail(TP_ERR_INVALID, "tp_ipc_alloc: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return fail(TP_ERR_CUDA, std::string("tp_ipc_alloc: ") + cudaGetErrorString(e));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");
  std::memcpy(handle_out, &h, sizeof(h));
  *ptr = p;
  return TP_OK;
}

int tp_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return fail(TP_ERR_INVALID, "tp_ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(TP_ERR_CUDA, std::string("tp_ipc_open: ") + cudaGetErrorString(e));
  return TP_OK;
}

int tp_ipc_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return fail(TP_ERR_CUDA, std::string("tp_ipc_close: ") + cudaGetErrorString(e));
  return TP_OK;
}

int tp_ipc_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return fail(TP_ERR_CUDA, std::string("tp_ipc_free: ") + cudaGetErrorString(e));
  return TP_OK;
}

int tp_decode_attention_sharded(const tp_page_pool* pool, const tp_tail* tail, tp_state state, const int32_t* d_state,
                                const void* q, int32_t q_dtype, int32_t num_q_heads, float scale, void* out,
                                const tp_exchange* x, void* workspace, size_t workspace_bytes, void* stream) {
  if (!x) return fail(TP_ERR_INVALID, "tp_decode_attention_sharded: exchange is NULL");
  return run_attention(pool, tail, state, const_cast<int32_t*>(d_state), q, q_dtype, num_q_heads, scale, out,
                       nullptr, workspace, workspace_bytes, stream, nullptr, x);
}

int tp_decode_step_sharded(const tp_page_pool* pool, const tp_tail* tail, int32_t* d_state, const void* k_new,
                           const void* v_new, int32_t kv_dtype, int64_t head_stride, const void* q, int32_t q_dtype,
                           int32_t num_q_heads, float scale, void* out, const tp_exchange* x, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (!x) return fail(TP_ERR_INVALID, "tp_decode_step_sharded: exchange is NULL");
  const int st = check_step_args(pool, tail, d_state, k_new, v_new, kv_dtype, head_stride);
  if (st != TP_OK) return st;
  StepArgs a{k_new, v_new, head_stride};
  tp_state none = {0, 0, 0, 0};
  return run_attention(pool, tail, none, d_state, q, q_dtype, num_q_heads, scale, out, nullptr, workspace,
                       workspace_bytes, stream, &a, x);
}

// ----------------------------------------------------------------------------- no-allocation variant
// Scratch for tp_decode_attention_noalloc: a fixed array in this module's device memory,
// created when the library is loaded on a device and held there until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_workspace[TP_NOALLOC_WORKSPACE_BYTES];

static std::mutex g_noalloc_mutex;
static void* g_noalloc_ptr[64] = {};  // device address of the array, per device ordinal

// Device address of the scratch array on the current device, resolved once per device with that
// device current (the host-side name of the array is not a device address).
static int noalloc_scratch(const char* who, void** ws) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(TP_ERR_CUDA, std::string(who) + ": " + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(TP_ERR_UNSUPPORTED, std::string(who) + ": device ordinal above 63");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_workspace);
    if (e != cudaSuccess) return fail(TP_ERR_CUDA, std::string(who) + ": cudaGetSymbolAddress: " + cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *ws = g_noalloc_ptr[dev];
  return TP_OK;
}

int tp_decode_attention_noalloc(const tp_page_pool* pool, const tp_tail* tail, tp_state state, const int32_t* d_state,
                                const void* q, int32_t q_dtype, int32_t num_q_heads, float scale, void* out,
                                float* partial_out, void* stream) {
  if (!pool) return fail(TP_ERR_INVALID, "page pool is NULL");
  const size_t need = tp_decode_attention_workspace_size(pool->num_kv_heads, num_q_heads);
  if (need == 0) return fail(TP_ERR_INVALID, "num_q_heads must be divisible by num_kv_heads for GQA");
  if (need > sizeof(g_noalloc_workspace))
    return fail(TP_ERR_INVALID, "tp_decode_attention_noalloc: this head layout needs " + std::to_string(need) +
                                    " bytes of scratch, above the fixed " +
                                    std::to_string(sizeof(g_noalloc_workspace)) + "-byte maximum");
  void* ws = nullptr;
  const int st = noalloc_scratch("tp_decode_attention_noalloc", &ws);
  if (st != TP_OK) return st;
  // Word 0 of the scratch is the sticky stage-wait error word; start this call from zero.
  const cudaError_t e = cudaMemsetAsync(ws, 0, sizeof(int), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(TP_ERR_CUDA, std::string("tp_decode_attention_noalloc: ") + cudaGetErrorString(e));
  return tp_decode_attention(pool, tail, state, d_state, q, q_dtype, num_q_heads, scale, out, partial_out, ws,
                             sizeof(g_noalloc_workspace), stream);
}

int tp_noalloc_error(int32_t* error_out, void* stream) {
  if (!error_out) return fail(TP_ERR_INVALID, "tp_noalloc_error: error_out is NULL");
  void* ws = nullptr;
  const int st = noalloc_scratch("tp_noalloc_error", &ws);
  if (st != TP_OK) return st;
  int32_t word = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&word, ws, sizeof(word), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail(TP_ERR_CUDA, std::string("tp_noalloc_error: ") + cudaGetErrorString(e));
  *error_out = word;
  return TP_OK;
}

int tp_combine_partials(const float* partials, int32_t n_parts, int32_t num_q_heads, void* out, void* stream) {
  if (!partials || !out || n_parts <= 0 || num_q_heads <= 0) return fail(TP_ERR_INVALID, "tp_combine_partials: bad argument");
  combine_kernel<<<num_q_heads, kD, 0, static_cast<cudaStream_t>(stream)>>>(partials, n_parts, num_q_heads,
                                                                             static_cast<__half*>(out));
  return check_launch("tp_combine_partials");
}

}  // extern "C"
