/*
 * am_q4.h — C ABI of the B200 Q4 KV-cache attention library (libamq4.so).
 *
 * Plain C: pointers, sizes and small POD structs, no C++ or torch types.  Every
 * pointer named *device* is a CUDA device address on the current device; `stream`
 * is a cudaStream_t passed as void* (NULL = legacy default stream).  The library
 * allocates no device memory at run time: the caller owns the cache, the queries, the
 * outputs and the workspace.  The only device memory the library itself holds is one
 * fixed array of AM_STATIC_DECODE_SCRATCH_BYTES per device that loads it (the scratch of
 * am_q4_decode_noalloc), reserved when the library's module is loaded on that device.
 * Calls are stream-ordered and never synchronise the device.  Every function returns
 * AM_OK or a negative AM_ERR_* code; am_last_error() describes the last failure on the
 * calling thread.  There is no CPU fallback: an unsupported shape returns
 * AM_ERR_UNSUPPORTED.
 *
 * Each entry point names the reference interface it replaces (paths relative to the
 * agent-memory repository).
 */
#ifndef AM_Q4_H
#define AM_Q4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AM_ABI_VERSION 4

enum {
  AM_OK = 0,
  AM_ERR_INVALID = -1,     /* null pointer, bad shape, misaligned buffer, bad enum */
  AM_ERR_UNSUPPORTED = -2, /* no kernel for this head-dim / dtype combination */
  AM_ERR_WORKSPACE = -3,   /* workspace smaller than the call's *_workspace_bytes() */
  AM_ERR_CUDA = -4         /* a CUDA launch failed; see am_last_error() */
};

enum { AM_DTYPE_F16 = 0, AM_DTYPE_BF16 = 1, AM_DTYPE_F32 = 2, AM_DTYPE_U8 = 3 };
enum { AM_LAYOUT_CONTIGUOUS = 0, AM_LAYOUT_PAGED = 1 };
enum { AM_MASK_NONE = 0, AM_MASK_BOOL = 1, AM_MASK_ADDITIVE = 2 };

/* Bits a kernel ORs into the optional device status word. */
enum {
  AM_STATUS_BAD_BLOCK = 1,    /* a block-table entry outside [0, num_blocks) was skipped */
  AM_STATUS_BAD_POSITION = 2, /* a position outside the cache capacity was skipped */
  AM_STATUS_TIMEOUT = 4,      /* a bounded wait inside a kernel gave up */
  AM_STATUS_POOL_EXHAUSTED = 8 /* am_block_reserve: not enough free blocks, nothing taken */
};

/*
 * A Q4 KV cache: for K and V, packed 4-bit codes (8 per uint32, element d of a row in
 * word d/8 at bits 4*(d%8)), plus one scale and one bias per 64 elements (fp16 or bf16).
 *
 * AM_LAYOUT_CONTIGUOUS — the reference's BatchQuantizedKVCache tensors
 *   (mlx_quantized_extensions.py:243-248): codes [batch, n_kv_heads, capacity, dim/8],
 *   scales/biases [batch, n_kv_heads, capacity, dim/64].
 * AM_LAYOUT_PAGED — a block pool: codes [capacity(=num_blocks), n_kv_heads,
 *   block_tokens, dim/8] (scales/biases likewise), sequence b's position t lives in
 *   block block_table[b * block_table_stride + t / block_tokens].  Block accounting
 *   mirrors BlockPool (domain/services.py:31-450) with 256-token blocks
 *   (domain/entities.py:17).
 * Code rows must be 16-byte aligned (dim/8 words is always a multiple of 4).
 */
typedef struct am_q4_cache {
  uint32_t* k_codes;
  void* k_scales;
  void* k_biases;
  uint32_t* v_codes;
  void* v_scales;
  void* v_biases;
  int32_t scale_dtype;        /* AM_DTYPE_F16 or AM_DTYPE_BF16 */
  int32_t layout;             /* AM_LAYOUT_* */
  int32_t n_kv_heads;
  int32_t k_dim;              /* multiple of 64 */
  int32_t v_dim;              /* multiple of 64 */
  int32_t block_tokens;       /* paged: tokens per block, multiple of 16 */
  int64_t capacity;           /* contiguous: rows per (sequence, head); paged: num_blocks */
  int32_t batch;              /* contiguous: leading extent of the buffers */
  int32_t block_table_stride; /* paged: entries per block-table row */
  const int32_t* block_table; /* paged, device: [rows, block_table_stride] */
} am_q4_cache;

/*
 * One attention call: queries [batch, n_q_heads, q_len, k_dim] -> out [batch, n_q_heads,
 * q_len, v_dim] (last dims contiguous, other strides in elements).  Query l of sequence b
 * sits at cache position kv_len[b] - q_len + l; it sees key r when
 *   kv_start[b] <= r  and  (!causal or r <= pos)  and  (window <= 0 or r > pos - window)
 * and, if a dense mask is given, mask[b,h,l,r] keeps it (AM_MASK_BOOL, u8 != 0) or adds
 * to its score (AM_MASK_ADDITIVE, dtype mask_dtype).  Masked keys inside [0, kv_len)
 * take the finite minimum score, as the reference's where(mask, s, finfo.min) does
 * (mlx_fused_attention.py:95-100); positions >= kv_len do not exist.
 */
typedef struct am_attn_args {
  const void* q;
  int32_t q_dtype;            /* AM_DTYPE_F16 or AM_DTYPE_BF16 */
  int32_t batch;
  int32_t n_q_heads;          /* multiple of cache->n_kv_heads */
  int32_t q_len;
  int64_t q_stride_b, q_stride_h, q_stride_l;
  void* out;
  int32_t out_dtype;          /* AM_DTYPE_F16, AM_DTYPE_BF16 or AM_DTYPE_F32 */
  int32_t causal;
  int64_t o_stride_b, o_stride_h, o_stride_l;
  float scale;                /* softmax scale applied to q.k */
  int32_t window;             /* sliding window (0 = none) */
  const int32_t* kv_len;      /* device [batch] */
  const int32_t* kv_start;    /* device [batch] or NULL (left padding) */
  int32_t max_kv_len;         /* host upper bound of kv_len[] (sizes the grid) */
  int32_t mask_kind;          /* AM_MASK_* */
  const void* mask;           /* device, element strides below (0 = broadcast) */
  int32_t mask_dtype;         /* additive: AM_DTYPE_F16/BF16/F32; bool: AM_DTYPE_U8 */
  int32_t reserved0;
  int64_t mask_stride_b, mask_stride_h, mask_stride_l, mask_stride_n;
  int32_t* status;            /* device word or NULL: kernels OR AM_STATUS_* bits into it */
  /* Attention sinks (replaces the fp16 detour of mlx_sink_compat.py:46-69): device fp32
   * [n_q_heads] logits in scaled-score units, or NULL.  Each joins its head's softmax
   * normaliser as one extra key that carries no value. */
  const float* sinks;
} am_attn_args;

/* Library ABI version (AM_ABI_VERSION). */
int am_abi_version(void);

/* Description of the last error on this thread ("" when none). */
const char* am_last_error(void);

/*
 * mx.quantize(x, group_size=64, bits=4) over `rows` contiguous rows of `dim` elements
 * (replaces mlx_quantized_extensions.py:273-274, batch_engine.py:1948-1949,
 * safetensors_cache_adapter.py:177-178).  x: device fp16/bf16 [rows, dim];
 * codes [rows, dim/8]; scales/biases [rows, dim/64] in x's dtype.
 */
int am_q4_quantize(const void* x, int32_t dtype, int64_t rows, int32_t dim, uint32_t* codes,
                   void* scales, void* biases, void* stream);

/*
 * mx.dequantize (replaces mlx_sink_compat.py:46-57): out[r, d] = code * scale + bias,
 * written as out_dtype (F16, BF16 or F32).
 */
int am_q4_dequantize(const uint32_t* codes, const void* scales, const void* biases,
                     int32_t scale_dtype, int64_t rows, int32_t dim, void* out,
                     int32_t out_dtype, void* stream);

/*
 * Quantize-on-append (replaces BatchQuantizedKVCache.update_and_fetch,
 * mlx_quantized_extensions.py:224-306, and mlx-lm QuantizedKVCache.update_and_fetch):
 * quantizes k [batch, n_kv_heads, n_new, k_dim] and v [..., v_dim] (fp16/bf16, strides in
 * elements, last dim contiguous) and writes token l of sequence b to cache position
 * positions[b] + l, through the block table for a paged cache.  `dtype` must equal
 * cache->scale_dtype (scales keep the input dtype).  Out-of-range block ids or positions
 * are skipped and flagged in *status.
 */
int am_q4_append(const am_q4_cache* cache, const void* k, const void* v, int32_t dtype,
                 int32_t batch, int32_t n_new, int64_t k_stride_b, int64_t k_stride_h,
                 int64_t k_stride_l, int64_t v_stride_b, int64_t v_stride_h,
                 int64_t v_stride_l, const int32_t* positions, int32_t* status, void* stream);

/*
 * Workspace sizing (bytes; 0 = none needed).  am_q4_decode_workspace_bytes: the split-KV
 * partials of am_q4_decode.  am_q4_prefill_workspace_bytes: the fp16 rows of the keys and
 * values a prefill call can see (batch x n_kv_heads x span x (k_dim + v_dim) x 2 bytes, the
 * span being max_kv_len, or window + q_len - 1 with a sliding window; k_dim x 2 bytes per
 * row for k_dim 192 / v_dim 128, whose values the attention kernel dequantizes itself).
 * am_q4_attention_workspace_bytes: what am_q4_attention needs for the kernel it dispatches
 * to.  The reference's compiled path allocates its intermediates inside mlx
 * (mlx_fused_attention.py:86-109); here the caller owns that memory.
 */
size_t am_q4_decode_workspace_bytes(const am_q4_cache* cache, const am_attn_args* args);
size_t am_q4_prefill_workspace_bytes(const am_q4_cache* cache, const am_attn_args* args);
size_t am_q4_attention_workspace_bytes(const am_q4_cache* cache, const am_attn_args* args);

/*
 * Split-KV decode attention (replaces the L=1 path of _patched_q4_sdpa,
 * mlx_fused_attention.py:396-484, and the compiled quantized SDPA at :69-139 for small
 * q_len): requires n_rep * q_len <= 64 (n_rep = n_q_heads / n_kv_heads).
 */
int am_q4_decode(const am_q4_cache* cache, const am_attn_args* args, void* workspace,
                 size_t workspace_bytes, void* stream);

/*
 * Split-KV decode for callers that cannot allocate device memory (no counterpart in the
 * reference, whose attention path never takes a caller-provided workspace).  Same
 * arguments, checks and results as am_q4_decode, but the per-split scratch comes from one
 * array of AM_STATIC_DECODE_SCRATCH_BYTES compiled into the library and held on every GPU
 * that loads it until exit; calls needing more scratch return AM_ERR_WORKSPACE.  Nothing
 * is allocated.  All calls share that scratch: calls that overlap on the GPU race and must
 * be serialized by the caller.  The first call on a device looks the array's address up
 * (cudaGetSymbolAddress) with that device current; make it before any stream capture.
 */
#define AM_STATIC_DECODE_SCRATCH_BYTES (16u << 20)
int am_q4_decode_noalloc(const am_q4_cache* cache, const am_attn_args* args, void* stream);

/*
 * Chunked prefill attention on tcgen05 tensor cores (replaces the L>1 compiled path of
 * _fused_q4_sdpa, mlx_fused_attention.py:144-207, as driven by chunked prefill,
 * batch_engine.py:339-456).  Head dims (k_dim, v_dim): (64, 64), (128, 128), (128, 64),
 * (192, 128), (256, 256).  Two launches on `stream`: the keys and values the query block
 * can see are dequantized once into fp16 rows of `workspace` (256-byte aligned, at least
 * am_q4_prefill_workspace_bytes), then the attention kernel streams them to the tensor
 * cores (for (192, 128) only the keys: that kernel dequantizes the values from the cache
 * itself).  Dequantized values beyond fp16's range saturate at +-65504.
 */
int am_q4_prefill(const am_q4_cache* cache, const am_attn_args* args, void* workspace,
                  size_t workspace_bytes, void* stream);

/*
 * am_q4_prefill in two parts, so a serving loop can dequantize a layer's cached prefix
 * ahead of time (on another stream, while the previous layer's attention runs) and only
 * the newly appended chunk on the layer's critical path.  The reference has no such split:
 * its chunked prefill (batch_engine.py:339-456) hands the whole Q4 cache to the compiled
 * quantized SDPA (mlx_fused_attention.py:144-207), which dequantizes inside the call.
 *
 * am_q4_prefill_stage: the stage kernel alone, writing into `workspace` the fp16 rows of
 * the visible keys (and values) at positions [key_lo, key_hi) of every sequence (rows of
 * other positions are left untouched; positions from kv_len up to the attention kernel's
 * last key tile, which ends before max_kv_len + 128, are written as zeros, and later rows,
 * which no attention call reads, are not written).  `args` describe the attention call the rows are for (the same
 * batch, q_len, kv_len, kv_start, window, mask kind and max_kv_len as the later
 * am_q4_prefill_attend); its query and output pointers are not read.
 * am_q4_prefill_attend: the attention kernel alone, over a workspace in which stage calls
 * covering [0, INT_MAX) together (e.g. [0, prefix) then [prefix, INT_MAX)) have written
 * every row since the cache last changed.  Stage + attend over the same workspace give
 * exactly the outputs of am_q4_prefill.
 */
int am_q4_prefill_stage(const am_q4_cache* cache, const am_attn_args* args, int32_t key_lo,
                        int32_t key_hi, void* workspace, size_t workspace_bytes, void* stream);
int am_q4_prefill_attend(const am_q4_cache* cache, const am_attn_args* args, void* workspace,
                         size_t workspace_bytes, void* stream);

/*
 * quantized_scaled_dot_product_attention (mlx_fused_attention.py:462-484): dispatches to
 * am_q4_decode for short query blocks and am_q4_prefill otherwise.
 */
int am_q4_attention(const am_q4_cache* cache, const am_attn_args* args, void* workspace,
                    size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- paged pool blocks
 *
 * `pool` describes a paged cache (layout AM_LAYOUT_PAGED; capacity = num_blocks; the
 * block table is not used by these calls).  Device arrays throughout. */

/*
 * Copy whole blocks between the pool and a packed byte buffer laid out like the
 * reference's persisted block tensors (replaces the per-block mx arrays written and read
 * by safetensors_cache_adapter.py:141-199, :284-327): block i contributes six tensors
 * [1, n_kv_heads, tokens[i], cols] -- K weights (uint32, cols = k_dim/8), K scales,
 * K biases (scale dtype, cols = k_dim/64), V weights, V scales, V biases -- at byte
 * offsets offsets[6*i .. 6*i+5] of the buffer.  pack: pool -> buffer; unpack: buffer ->
 * pool.  Bad block ids or token counts are skipped and flagged AM_STATUS_BAD_BLOCK.
 */
int am_q4_blocks_pack(const am_q4_cache* pool, const int32_t* block_ids, const int32_t* tokens,
                      const int64_t* offsets, int32_t n_blocks, void* buffer, int32_t* status,
                      void* stream);
int am_q4_blocks_unpack(const am_q4_cache* pool, const int32_t* block_ids, const int32_t* tokens,
                        const int64_t* offsets, int32_t n_blocks, const void* buffer,
                        int32_t* status, void* stream);

/*
 * The pool's free list on the device (replaces BlockPool.allocate / free,
 * domain/services.py:111-223, for growth inside a captured step).  free_ids[0, *free_top)
 * is the stack of free block ids, top last.
 * am_block_reserve: for every row r, entries [0, ceil((lengths[r] + add[r]) /
 * block_tokens)) of table row r that are < 0 take the next id from the top, rows in
 * order, entries in order; all-or-nothing (AM_STATUS_POOL_EXHAUSTED).
 * am_block_release: entries [keep_blocks[r], table_stride) of row r that hold a block go
 * back onto the stack in row-major order and become -1; a release that would overflow the
 * stack changes nothing and sets AM_STATUS_BAD_BLOCK.
 */
int am_block_reserve(int32_t* free_ids, int32_t* free_top, int32_t num_blocks, int32_t* table,
                     int32_t table_stride, int32_t rows, const int32_t* lengths,
                     const int32_t* add, int32_t block_tokens, int32_t* status, void* stream);
int am_block_release(int32_t* free_ids, int32_t* free_top, int32_t num_blocks, int32_t* table,
                     int32_t table_stride, int32_t rows, const int32_t* keep_blocks,
                     int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AM_Q4_H */
