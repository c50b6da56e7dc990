/*
 * turbopolar.h -- C ABI of libturbopolar.so, the B200 (sm_100a) implementation of
 * TurboPolar's compressed-KV single-batch decode path.
 *
 * The reference (dawsonblock/Turbopolar) runs this path through MLX on Apple GPUs.  Each
 * entry point below replaces one reference interface, cited as path:line inside that
 * project.  Conventions shared by every entry point:
 *
 *   - Plain pointers and sizes only.  Device pointers are CUDA global-memory addresses on
 *     the current device; `stream` is a cudaStream_t passed as void*.
 *   - Nothing allocates except tp_ipc_alloc, the one allocation helper (it creates a
 *     sequence-sharding exchange buffer that other processes map; it is called once at set-up,
 *     never on the decode path): every buffer (page pools, tail, state words, workspace,
 *     outputs) belongs to the caller.  Every launch is asynchronous on `stream`.
 *   - The return value is a tp_status; on failure tp_last_error() returns a message for
 *     the calling thread.  TP_ERR_INVALID maps to Python ValueError, TP_ERR_UNSUPPORTED to
 *     NotImplementedError, TP_ERR_CUDA to RuntimeError.
 *   - Batch size 1, head_dim 128, block (page) size 64 tokens, grouped int8 values with 32
 *     channels per group: the reference's supported contract
 *     (rfsn_v11/candidates/turbo_polar_config.py:27-55).
 */
#ifndef TURBOPOLAR_H_
#define TURBOPOLAR_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TP_HEAD_DIM 128
#define TP_PAGE_TOKENS 64
#define TP_V_GROUP 32
/* Floats per partial record: m (log2 domain), l, then 128 unnormalised outputs. */
#define TP_PARTIAL_FLOATS 130

typedef enum tp_status {
  TP_OK = 0,
  TP_ERR_INVALID = 1,     /* bad argument or state (ValueError) */
  TP_ERR_UNSUPPORTED = 2, /* outside the supported contract (NotImplementedError) */
  TP_ERR_CUDA = 3         /* launch / runtime failure (RuntimeError) */
} tp_status;

typedef enum tp_dtype { TP_F16 = 0, TP_F32 = 1 } tp_dtype;

/* Key format: the fields of TurboPolarConfig that shape a PolarKeyBlock
 * (rfsn_v11/candidates/turbo_polar_config.py:11-21, rfsn_v11/quant/polar/encoder.py:24-98). */
typedef struct tp_format {
  int32_t l1_bits;    /* k_angle_bits_level1: 4 or 8 */
  int32_t deep_bits;  /* k_angle_bits_deep: 2, 4 or 8 */
  int32_t split_dim;  /* even, 0..128: pairs [0, split_dim/2) use level-1 codes */
  int32_t int8_radii; /* 0: float16 radii; 1: log-int8 radii + one float16 scale per page */
} tp_format;

/* Device page pool in the kernels' layout: one contiguous page block per (KV head, page), made
 * of two "units" (half pages, tokens 0-31 and 32-63), so a decode kernel streams a half page
 * with one bulk copy.  A unit of tp_unit_bytes(fmt) bytes holds, in this order:
 *   radii     [32][64] float16 (int8 when fmt.int8_radii); float16 rows are XOR-swizzled:
 *             16-byte chunk c of row l is stored at chunk c ^ (l & 7)
 *   v_codes   4096 bytes, (code ^ 0x80) in mma fragment order
 *   codes     [32][l1_row + deep_row]: each token row holds its level-1 codes then its deep
 *             codes, each packed exactly as the reference packs them
 *   v_scales  [128] float16 in fragment order (one per token and 32-channel group)
 * The codes are the reference's block-storage codes (rfsn_v11/generation/storage.py:17-169)
 * bit for bit; only their placement differs.  tp_export_pages / tp_import_pages convert to and
 * from the reference layout (tp_block_store).  Fields:
 *   pages         [H_kv][page_capacity][2 * tp_unit_bytes(fmt)] bytes, 16-byte aligned
 *   radii_scales  [H_kv][page_capacity] float16 (fmt.int8_radii only, else NULL) */
typedef struct tp_page_pool {
  void* pages;
  void* radii_scales;
  int32_t num_kv_heads;
  int32_t page_capacity;
  tp_format fmt;
} tp_page_pool;

/* Pages in the reference's block-storage layout (rfsn_v11/generation/storage.py:89-102 and
 * :160-169), one array per field with every page of a head contiguous:
 *   radii            [H_kv][page_capacity][64][64]  float16 (int8 when fmt.int8_radii), row-major
 *   radii_scales     [H_kv][page_capacity]          float16 (fmt.int8_radii only, else NULL)
 *   angle_codes_l1   [H_kv][page_capacity][64][l1_row_bytes]   uint8
 *   angle_codes_deep [H_kv][page_capacity][64][deep_row_bytes] uint8
 *   v_codes          [H_kv][page_capacity][64][128] int8
 *   v_scales         [H_kv][page_capacity][64][4]   float16
 * Key fields may all be NULL (values only).  Row byte counts come from tp_row_bytes(). */
typedef struct tp_block_store {
  void* radii;
  void* radii_scales;
  void* angle_codes_l1;
  void* angle_codes_deep;
  void* v_codes;
  void* v_scales;
  int32_t num_kv_heads;
  int32_t page_capacity;
  tp_format fmt;
} tp_block_store;

/* Dense tail (the reference's partial block, rfsn_v11/generation/turbo_polar_cache.py:110-126):
 * k and v are [H_kv][64][128] in `dtype`, the first tail_len token rows valid. */
typedef struct tp_tail {
  void* k;
  void* v;
  int32_t dtype; /* tp_dtype */
} tp_tail;

/* Cache state.  Kernels that take `const int32_t* d_state` read these four words from
 * device memory when the pointer is non-NULL (CUDA-graph replay) and from the struct
 * passed by value otherwise.  Word order: n_pages, tail_len, seq_len, first_page, then
 * an error word written by tp_append and a ticket word it uses internally (both zero at
 * rest).  first_page is the absolute index of local page 0 (non-zero on sequence shards);
 * token l of local page p sits at absolute position (first_page + p) * 64 + l, tail token
 * t at (first_page + n_pages) * 64 + t, and positions >= seq_len are masked
 * (rfsn_v11/kernels/turbo_polar/metal.py:317-319). */
typedef struct tp_state {
  int32_t n_pages;
  int32_t tail_len;
  int32_t seq_len;
  int32_t first_page;
} tp_state;
#define TP_STATE_WORDS 6

/* Bytes per token row of the level-1 and deep code arrays for `fmt`
 * (tests/benchmarks/test_turbo_polar_offline.py:26-34).  Returns TP_ERR_UNSUPPORTED for a
 * format outside turbo_polar_config.py / encoder.py's accepted bit widths. */
int tp_row_bytes(const tp_format* fmt, int32_t* l1_row_bytes, int32_t* deep_row_bytes);

/* Bytes of one unit (half page of one KV head) of a tp_page_pool in format `fmt`: the
 * reference's block payload per 32 tokens without the radius scale (296 x 32 = 9472 for the
 * default format; rfsn_v11/generation/turbo_polar_cache.py:154-161 counts the same bytes). */
int tp_unit_bytes(const tp_format* fmt, int32_t* unit_bytes);

/* Encode n_pages full 64-token blocks of dense keys/values into pool pages
 * [dst_page, dst_page + n_pages) of every KV head.  Token t of head h of the source is at
 * k + (h * head_stride + (src_token0 + t) * token_stride) elements (innermost 128 contiguous),
 * same for v.  Bit-exact with PolarQuantEncoder.encode_block + GroupedVQuantizer.quantize_block
 * (rfsn_v11/quant/polar/encoder.py:24-130, rfsn_v11/quant/v_quant/encoder.py:16-30) as called
 * by TurboPolarKVCacheRuntime._flush_block (rfsn_v11/generation/turbo_polar_cache.py:128-161).
 * If d_state is non-NULL, n_pages is added to its n_pages word and 64*n_pages to seq_len after
 * the encode (used when a long append encodes whole pages straight from its input). */
int tp_encode_pages(const tp_page_pool* pool, const void* k, const void* v, int32_t dtype,
                    int64_t head_stride, int64_t token_stride, int64_t src_token0,
                    int32_t n_pages, int32_t dst_page, int32_t* d_state, void* stream);

/* Append n_tokens (1..64) tokens to the dense tail at the device-side tail_len; when the
 * tail reaches 64 tokens, encode it into page n_pages and empty it; then advance the state
 * words (TurboPolarKVCacheRuntime.append, rfsn_v11/generation/turbo_polar_cache.py:106-126).
 * The caller keeps tail_len + n_tokens <= 64.  A violated bound or a full pool sets the
 * state's error word (1: tail overflow, 2: page pool full) and changes nothing else. */
int tp_append(const tp_page_pool* pool, const tp_tail* tail, int32_t* d_state, const void* k_new,
              const void* v_new, int32_t dtype, int64_t head_stride, int64_t token_stride,
              int32_t n_tokens, void* stream);

/* Workspace bytes tp_decode_attention needs for this head layout.  The workspace must be
 * zero-filled once when allocated; every launch leaves its counters at zero again. */
size_t tp_decode_attention_workspace_size(int32_t num_kv_heads, int32_t num_q_heads);

/* Fused decode attention over compressed pages plus the dense tail, for one query token:
 *   out[hq][:] = softmax_t(scale * q[hq] . K[hq / G][t]) @ V[hq / G]     (fp16, [H_q][128])
 * Replaces MetalKernelBridge.execute_online_attention_quant_v_dense_tail and
 * execute_online_attention_quant_v (rfsn_v11/kernels/turbo_polar/metal.py:651-792, kernels
 * tqpolar_online_attention.metal:197-629) with the reference's CPU fallback as the numeric
 * target (metal.py:267-332).  q is [H_q][128] in q_dtype (float32 queries are rounded to
 * float16 as the reference's kernels read them).  With partial_out non-NULL the kernel
 * writes, instead of `out`, one unnormalised partial per query head
 * [H_q][TP_PARTIAL_FLOATS] = (m in log2 units, l, o[128]) for a cross-shard log-sum-exp
 * merge (tp_combine_partials).  `state` is used when d_state is NULL.  When the previous call
 * of this library on `stream` writes no buffer this call reads (another cache and another
 * query), this call's page pass starts streaming before that call's kernels have completed;
 * the library compares the buffers' addresses itself. */
int tp_decode_attention(const tp_page_pool* pool, const tp_tail* tail, tp_state state,
                        const int32_t* d_state, const void* q, int32_t q_dtype,
                        int32_t num_q_heads, float scale, void* out, float* partial_out,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Fused decode attention over compressed keys and dense float16 values.  Replaces
 * MetalKernelBridge.execute_online_attention_dense_v (rfsn_v11/kernels/turbo_polar/
 * metal.py:587-649, kernel tqpolar_online_attention.metal:10-195; numeric target its CPU
 * fallback, metal.py:267-291): the keys of pool pages [0, state.n_pages) (their value codes
 * are not read), the values v[h][t][:] of KV head h and token t = 64 * page + row, heads
 * v_head_stride elements apart (a multiple of 8, >= 128 * v_tokens; v 16-byte aligned), tokens
 * t >= state.seq_len masked.  state.tail_len and state.first_page must be 0 and
 * 1 <= seq_len <= min(64 * n_pages, v_tokens); values past v_tokens read as zero.  Other
 * arguments, the workspace and the output as tp_decode_attention. */
int tp_decode_attention_dense_v(const tp_page_pool* pool, tp_state state, const void* v,
                                int64_t v_head_stride, int64_t v_tokens, const void* q,
                                int32_t q_dtype, int32_t num_q_heads, float scale, void* out,
                                float* partial_out, void* workspace, size_t workspace_bytes,
                                void* stream);

/* One decode step in one call: append one token per KV head, then attend over everything
 * including it.  Replaces TurboPolarFastCache.decode_attention
 * (benchmarks/turbopolar_fast_attention.py:106-188), i.e. TurboPolarKVCacheRuntime.append
 * (rfsn_v11/generation/turbo_polar_cache.py:106-161) followed by the fused attention above,
 * with the same results as tp_append + tp_decode_attention.  k_new / v_new hold token rows
 * [H_kv][128] in kv_dtype (the tail's dtype), heads head_stride elements apart (16-byte
 * aligned rows).  The state words d_state (required) are read at the start and advanced by
 * the call on the device; when the token completes the tail's page, the page is encoded into
 * pool page n_pages first.  A full pool drops the token and sets d_state[4] = 2. */
int tp_decode_step(const tp_page_pool* pool, const tp_tail* tail, int32_t* d_state,
                   const void* k_new, const void* v_new, int32_t kv_dtype, int64_t head_stride,
                   const void* q, int32_t q_dtype, int32_t num_q_heads, float scale, void* out,
                   float* partial_out, void* workspace, size_t workspace_bytes, void* stream);

/* Size of the fixed scratch array behind tp_decode_attention_noalloc (2 MiB per device). */
#define TP_NOALLOC_WORKSPACE_BYTES (2u * 1024u * 1024u)

/* tp_decode_attention without a caller-provided workspace, for callers that cannot allocate
 * device memory: a plugin inside a host runtime that owns every allocation, code that runs
 * while a stream is being captured (cudaMalloc is not permitted there), or a latency-critical
 * path that must not take the allocator's locks.  No counterpart in the reference (its MLX
 * bridge allocates through MLX on every call).  Scratch is a fixed TP_NOALLOC_WORKSPACE_BYTES
 * array in the library's device memory on every GPU that loads the library, kept until the
 * process exits; layouts needing more (tp_decode_attention_workspace_size) are rejected with
 * TP_ERR_INVALID.  The first call on a device resolves the array's address with that device
 * current, so make it before capturing a stream.  Every call on a device shares the one
 * array: calls whose executions overlap on the GPU (concurrent streams) race and must be
 * serialised by the caller.  Allocates nothing (no cudaMalloc / cudaFree).  Each call clears
 * the array's error word (word 0) before it launches; tp_noalloc_error reads it back. */
int tp_decode_attention_noalloc(const tp_page_pool* pool, const tp_tail* tail, tp_state state,
                                const int32_t* d_state, const void* q, int32_t q_dtype,
                                int32_t num_q_heads, float scale, void* out, float* partial_out,
                                void* stream);

/* The error word of the last tp_decode_attention_noalloc call on the current device: 0, or 1
 * when a stage wait ran out (the output of that call is unusable).  Waits for `stream`, then
 * copies the word into *error_out.  The word plays the part that workspace word 0 plays for
 * tp_decode_attention, whose caller owns the workspace and can read it; a no-allocation caller
 * has no handle on the array, and the next call clears the word.  Allocates nothing.  No
 * counterpart in the reference. */
int tp_noalloc_error(int32_t* error_out, void* stream);

/* Merge n_parts partial records per query head, laid out [n_parts][H_q][TP_PARTIAL_FLOATS]
 * (the all-gathered output of tp_decode_attention on each sequence shard), into fp16
 * out[H_q][128]: M = max m_r, L = sum l_r 2^(m_r - M), O = sum o_r 2^(m_r - M) / L. */
int tp_combine_partials(const float* partials, int32_t n_parts, int32_t num_q_heads, void* out,
                        void* stream);

/* ---- Sequence sharding over the GPUs of one node, merged inside the attention launch.
 * No reference counterpart (the reference runs on one device).  Every rank holds a contiguous
 * page range of every KV head; its attention launch publishes each query head's partial
 * (m, l, o) into every rank's exchange buffer with peer stores over NVLink, as 64-bit words
 * that each carry one value and the call's epoch, waits (bounded, about a second) until every
 * rank's words of that head carry the epoch and merges them, so each rank writes the whole
 * fp16 output with no collective library call (tp_exchange_bytes sizes a buffer; allocate it
 * zero-filled, as tp_ipc_alloc does).  All ranks must
 * make the same sequence of sharded calls on their buffers (the buffers' epoch words advance
 * once per call).  A wait that runs out leaves workspace word 0 = 3 (the output is unusable). */
#define TP_MAX_RANKS 8

typedef struct tp_exchange {
  int32_t world, rank;            /* 2 <= world <= TP_MAX_RANKS */
  void* buffers[TP_MAX_RANKS];    /* rank r's exchange buffer as mapped in this process */
} tp_exchange;

/* Bytes of one rank's exchange buffer for `world` ranks and H_q query heads. */
size_t tp_exchange_bytes(int32_t world, int32_t num_q_heads);

/* Device memory another process can map: cudaMalloc'd, zeroed, with its 64-byte IPC handle
 * written to handle_out (tp_ipc_open maps it in a peer process). */
int tp_ipc_alloc(size_t bytes, void** ptr, void* handle_out);
int tp_ipc_open(const void* handle, void** ptr);
int tp_ipc_close(void* ptr);
int tp_ipc_free(void* ptr);

/* tp_decode_attention / tp_decode_step of one shard, merged across the ranks of `x` into
 * `out` (no partial output). */
int tp_decode_attention_sharded(const tp_page_pool* pool, const tp_tail* tail, tp_state state,
                                const int32_t* d_state, const void* q, int32_t q_dtype,
                                int32_t num_q_heads, float scale, void* out, const tp_exchange* x,
                                void* workspace, size_t workspace_bytes, void* stream);
int tp_decode_step_sharded(const tp_page_pool* pool, const tp_tail* tail, int32_t* d_state,
                           const void* k_new, const void* v_new, int32_t kv_dtype, int64_t head_stride,
                           const void* q, int32_t q_dtype, int32_t num_q_heads, float scale, void* out,
                           const tp_exchange* x, void* workspace, size_t workspace_bytes, void* stream);

/* Scores only: scores[hq][p*64 + l] = scale * q[hq] . K[hq / G][page p][l] for local pages
 * [0, n_pages), fp16 [H_q][n_pages*64].  Replaces MetalKernelBridge.execute_fused_qk
 * (rfsn_v11/kernels/turbo_polar/metal.py:494-530, tqpolar_fused_qk.metal:4-100); accumulates
 * in float32 where the Metal kernel used float16. */
int tp_fused_scores(const tp_page_pool* pool, int32_t n_pages, const void* q, int32_t q_dtype,
                    int32_t num_q_heads, float scale, void* scores, void* stream);

/* Decompress pages [first_page, first_page + n_pages) to dense fp16 keys and values,
 * k_out/v_out [H_kv][n_pages*64][128] (PolarQuantDecoder.decode_block and
 * GroupedVQuantizer.dequantize_block, rfsn_v11/quant/polar/decoder.py:7-67,
 * rfsn_v11/quant/v_quant/encoder.py:32-38; the prefill decompress-on-read path of
 * benchmarks/turbopolar_fast_attention.py:56-86). */
int tp_decode_pages(const tp_page_pool* pool, int32_t first_page, int32_t n_pages, void* k_out,
                    void* v_out, void* stream);

/* Copy pages [first_page, first_page + n_pages) of `pool` into pages [0, n_pages) of `ref`,
 * a block store of the same heads and format (storage.py:89-102 and :160-169), e.g. to serve
 * TurboPolarKVCacheRuntime.get_fused_attention_inputs
 * (rfsn_v11/generation/turbo_polar_cache.py:163-198).  With ref's key fields NULL only the
 * values are copied. */
int tp_export_pages(const tp_page_pool* pool, int32_t first_page, int32_t n_pages, const tp_block_store* ref,
                    void* stream);

/* The inverse: load reference-layout pages [0, n_pages) of `ref` into pool pages
 * [first_page, first_page + n_pages) (payloads handed to the bridge's execute_* calls,
 * rfsn_v11/kernels/turbo_polar/metal.py:651-792). */
int tp_import_pages(const tp_page_pool* pool, int32_t first_page, int32_t n_pages, const tp_block_store* ref,
                    void* stream);

/* Message of the last failed call on this thread ("" if none). */
const char* tp_last_error(void);

/* ABI version of this library. */
int tp_version(void);

#ifdef __cplusplus
}
#endif

#endif /* TURBOPOLAR_H_ */
