// C ABI of libamq4.so: argument validation, dispatch to the kernel launchers, and
// per-thread error reporting.  The library allocates no device memory and keeps no
// pointer after a call returns.
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdint>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include <cudaTypedefs.h>  // PFN_cuTensorMapEncodeTiled

#include <mutex>

#include "am_common.cuh"
#include "am_internal.h"

namespace am {

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

void clear_error() { g_last_error[0] = '\0'; }

static int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return AM_OK;
  if (e == cudaErrorNotSupported) {
    set_error("%s: no kernel for this configuration", what);
    return AM_ERR_UNSUPPORTED;
  }
  set_error("%s: CUDA error %d (%s)", what, static_cast<int>(e), cudaGetErrorString(e));
  return AM_ERR_CUDA;
}

static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

static bool valid_half_dtype(int d) { return d == AM_DTYPE_F16 || d == AM_DTYPE_BF16; }

static int check_cache(const am_q4_cache* c, const char* fn) {
  if (c == nullptr) {
    set_error("%s: cache is NULL", fn);
    return AM_ERR_INVALID;
  }
  if (!c->k_codes || !c->k_scales || !c->k_biases || !c->v_codes || !c->v_scales || !c->v_biases) {
    set_error("%s: a cache buffer is NULL", fn);
    return AM_ERR_INVALID;
  }
  if (!valid_half_dtype(c->scale_dtype)) {
    set_error("%s: scale_dtype must be F16 or BF16", fn);
    return AM_ERR_INVALID;
  }
  if (c->n_kv_heads <= 0 || c->k_dim <= 0 || c->v_dim <= 0 || c->k_dim % 64 || c->v_dim % 64) {
    set_error("%s: n_kv_heads > 0 and head dims that are multiples of 64 required (got %d, %d, %d)",
              fn, c->n_kv_heads, c->k_dim, c->v_dim);
    return AM_ERR_INVALID;
  }
  if (!aligned(c->k_codes, 16) || !aligned(c->v_codes, 16) || !aligned(c->k_scales, 4) ||
      !aligned(c->k_biases, 4) || !aligned(c->v_scales, 4) || !aligned(c->v_biases, 4)) {
    set_error("%s: codes must be 16-byte and scales/biases 4-byte aligned", fn);
    return AM_ERR_INVALID;
  }
  if (c->layout == AM_LAYOUT_CONTIGUOUS) {
    if (c->capacity <= 0 || c->capacity % 16) {
      set_error("%s: contiguous capacity must be a positive multiple of 16 (got %lld)", fn,
                static_cast<long long>(c->capacity));
      return AM_ERR_INVALID;
    }
  } else if (c->layout == AM_LAYOUT_PAGED) {
    if (c->block_table == nullptr || c->block_table_stride <= 0 || c->capacity <= 0 ||
        c->block_tokens <= 0 || c->block_tokens % 16) {
      set_error("%s: paged cache needs a block table, num_blocks > 0 and block_tokens %% 16 == 0", fn);
      return AM_ERR_INVALID;
    }
  } else {
    set_error("%s: unknown layout %d", fn, c->layout);
    return AM_ERR_INVALID;
  }
  return AM_OK;
}

static int check_args(const am_q4_cache* c, const am_attn_args* a, const char* fn) {
  if (a == nullptr || a->q == nullptr || a->out == nullptr || a->kv_len == nullptr) {
    set_error("%s: q, out and kv_len are required", fn);
    return AM_ERR_INVALID;
  }
  if (!valid_half_dtype(a->q_dtype)) {
    set_error("%s: q_dtype must be F16 or BF16", fn);
    return AM_ERR_INVALID;
  }
  if (!(valid_half_dtype(a->out_dtype) || a->out_dtype == AM_DTYPE_F32)) {
    set_error("%s: out_dtype must be F16, BF16 or F32", fn);
    return AM_ERR_INVALID;
  }
  if (a->batch < 0 || a->n_q_heads <= 0 || a->q_len < 0 || a->n_q_heads % c->n_kv_heads) {
    set_error("%s: n_q_heads (%d) must be a positive multiple of n_kv_heads (%d)", fn,
              a->n_q_heads, c->n_kv_heads);
    return AM_ERR_INVALID;
  }
  if (c->layout == AM_LAYOUT_CONTIGUOUS && a->batch > c->batch) {
    set_error("%s: batch %d exceeds the cache's batch extent %d", fn, a->batch, c->batch);
    return AM_ERR_INVALID;
  }
  if (a->max_kv_len < 0) {
    set_error("%s: max_kv_len must be >= 0", fn);
    return AM_ERR_INVALID;
  }
  if (a->mask_kind != AM_MASK_NONE) {
    if (a->mask == nullptr) {
      set_error("%s: mask_kind set but mask is NULL", fn);
      return AM_ERR_INVALID;
    }
    if (a->mask_kind == AM_MASK_BOOL && a->mask_dtype != AM_DTYPE_U8) {
      set_error("%s: boolean masks are u8", fn);
      return AM_ERR_INVALID;
    }
    if (a->mask_kind == AM_MASK_ADDITIVE && !(valid_half_dtype(a->mask_dtype) ||
                                              a->mask_dtype == AM_DTYPE_F32)) {
      set_error("%s: additive masks are F16, BF16 or F32", fn);
      return AM_ERR_INVALID;
    }
    if (a->mask_kind != AM_MASK_BOOL && a->mask_kind != AM_MASK_ADDITIVE) {
      set_error("%s: unknown mask_kind %d", fn, a->mask_kind);
      return AM_ERR_INVALID;
    }
  }
  if (!std::isfinite(a->scale)) {
    set_error("%s: scale must be finite", fn);
    return AM_ERR_INVALID;
  }
  return AM_OK;
}

// Decode grid geometry: row groups of up to 8 query rows (n_rep * q_len rows per KV head)
// and the KV split.  The span of a windowed call is the window plus the query rows, plus
// up to one stage of keys from rounding the first key down to a stage boundary.
static int decode_geometry(const am_q4_cache* c, const am_attn_args* a, int* row_groups,
                           int* chunk, int* n_chunks, int* cluster) {
  const int n_rep = a->n_q_heads / c->n_kv_heads;
  const int rows = n_rep * a->q_len;
  *row_groups = (rows + 7) / 8;
  int span = a->max_kv_len;
  if (a->mask_kind == AM_MASK_NONE && a->window > 0) {
    const long long w = (long long)a->window + a->q_len - 1 + decode_stage_tokens(c->k_dim, c->v_dim) - 1;
    if (w < span) span = static_cast<int>(w);
  }
  decode_plan(a->batch, c->n_kv_heads, *row_groups, span, decode_ctas_per_sm(c->k_dim, c->v_dim),
              c->k_dim, c->v_dim, chunk, n_chunks, cluster);
  return rows;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against the
// driver library); null when the driver does not provide it.
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    } else {
      (void)cudaGetLastError();
    }
  });
  return fn;
}

// A 2-D map over a codes array seen as [rows, row_bytes] bytes; a box is box_bytes (32, 64
// or 128) of box_rows rows, swizzled by the box width; rows past the array read as zeros.
static bool encode_codes_map(CUtensorMap* m, const void* base, int64_t rows, int row_bytes,
                             int box_bytes, int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  const CUtensorMapSwizzle sw = box_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                : box_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                  : CU_TENSOR_MAP_SWIZZLE_32B;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_bytes), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t elem[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, elem,
             CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Decode kernels with 32-, 64- or 128-byte code rows (head dims 64, 128, 256; Dk = 192 as a
// 64-byte plus a 32-byte box) read K and V codes through swizzled tensor maps.
static bool decode_uses_tensor_maps(int k_dim, int v_dim) {
  auto ok = [](int d) { return d == 64 || d == 128 || d == 256; };
  return (ok(k_dim) || k_dim == 192) && ok(v_dim);
}

// Limit of the kernels' bounded waits.  AM_Q4_TEST_WAIT_LIMIT_NS (read on every call) lowers
// it for tests that drive the timeout path; 0 makes every pipeline wait give up at once (the
// kernels still let their copies in flight land before they return).  Unset, the limit is
// kWaitLimitNs.
static uint64_t wait_limit_ns() {
  const char* env = getenv("AM_Q4_TEST_WAIT_LIMIT_NS");
  if (env == nullptr || *env == '\0') return kWaitLimitNs;
  char* end = nullptr;
  const unsigned long long v = strtoull(env, &end, 10);
  return (end != env && v < kWaitLimitNs) ? static_cast<uint64_t>(v) : kWaitLimitNs;
}

static void fill_params(DecodeParams& p, const am_q4_cache* cache, const am_attn_args* a) {
  const int n_rep = a->n_q_heads / cache->n_kv_heads;
  p.wait_ns = wait_limit_ns();
  p.kc = cache->k_codes;
  p.ks = static_cast<const uint16_t*>(cache->k_scales);
  p.kb = static_cast<const uint16_t*>(cache->k_biases);
  p.vc = cache->v_codes;
  p.vs = static_cast<const uint16_t*>(cache->v_scales);
  p.vb = static_cast<const uint16_t*>(cache->v_biases);
  p.capacity = cache->capacity;
  p.table = cache->block_table;
  p.table_stride = cache->block_table_stride;
  p.block_tokens = cache->block_tokens;
  p.bt_shift = 0;
  while (cache->block_tokens > 0 && (1 << p.bt_shift) < cache->block_tokens) ++p.bt_shift;
  p.hkv = cache->n_kv_heads;
  p.k_dim = cache->k_dim;
  p.v_dim = cache->v_dim;
  p.hq = a->n_q_heads;
  p.q_len = a->q_len;
  p.n_rep = n_rep;
  p.rows_per_head = n_rep * a->q_len;
  p.q_bf16 = a->q_dtype == AM_DTYPE_BF16;
  p.q = static_cast<const uint16_t*>(a->q);
  p.qsb = a->q_stride_b;
  p.qsh = a->q_stride_h;
  p.qsl = a->q_stride_l;
  p.out = a->out;
  p.out_dtype = a->out_dtype;
  p.osb = a->o_stride_b;
  p.osh = a->o_stride_h;
  p.osl = a->o_stride_l;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.kv_len = a->kv_len;
  p.kv_start = a->kv_start;
  p.causal = a->causal;
  p.window = a->window;
  p.sinks = a->sinks;
  p.mask_kind = a->mask_kind;
  p.mask_dtype = a->mask_dtype;
  p.mask = a->mask;
  p.msb = a->mask_stride_b;
  p.msh = a->mask_stride_h;
  p.msl = a->mask_stride_l;
  p.msn = a->mask_stride_n;
  p.status = a->status;
}

// Workspace planes of a prefill call: nw rows per (sequence, KV head) hold the keys the query
// block can see, [lo, kv_len) -- the window plus the block when a sliding window applies
// (and no dense mask), else up to max_kv_len keys; K rows first, V rows 256-byte aligned
// after them (none for head dims whose attention kernel dequantizes V itself).
struct PrefillPlanes {
  int nw;
  int64_t rows;
  size_t k_bytes, v_bytes;
};

static PrefillPlanes prefill_planes(const am_q4_cache* c, const am_attn_args* a) {
  int64_t span = a->max_kv_len;
  if (a->mask_kind == AM_MASK_NONE && a->window > 0)
    span = std::min<int64_t>(span, static_cast<int64_t>(a->window) + a->q_len - 1);
  PrefillPlanes pl;
  pl.nw = static_cast<int>(std::max<int64_t>(8, (span + 7) / 8 * 8));
  pl.rows = static_cast<int64_t>(a->batch) * c->n_kv_heads * pl.nw;
  pl.k_bytes = (static_cast<size_t>(pl.rows) * c->k_dim * 2 + 255) / 256 * 256;
  pl.v_bytes = prefill_v_in_kernel(c->k_dim, c->v_dim) ? 0 : static_cast<size_t>(pl.rows) * c->v_dim * 2;
  return pl;
}

// am_q4_attention's dispatch: query blocks of more than 64 rows per KV head (n_rep * q_len),
// or of at least 16 positions, take the tcgen05 prefill kernel; shorter ones split-KV decode.
static bool routes_to_prefill(const am_q4_cache* c, const am_attn_args* a) {
  if (c == nullptr || a == nullptr || c->n_kv_heads <= 0 || a->n_q_heads <= 0) return false;
  const int n_rep = a->n_q_heads / c->n_kv_heads;
  return n_rep * a->q_len > 64 || (a->q_len >= 16 && prefill_supported(c->k_dim, c->v_dim));
}

}  // namespace am

using namespace am;

extern "C" {

int am_abi_version(void) { return AM_ABI_VERSION; }

const char* am_last_error(void) { return g_last_error; }

int am_q4_quantize(const void* x, int32_t dtype, int64_t rows, int32_t dim, uint32_t* codes,
                   void* scales, void* biases, void* stream) {
  clear_error();
  if (!valid_half_dtype(dtype) || rows < 0 || dim <= 0 || dim % 64) {
    set_error("am_q4_quantize: dtype F16/BF16 and dim %% 64 == 0 required (dim=%d)", dim);
    return AM_ERR_INVALID;
  }
  if (rows == 0) return AM_OK;
  if (!x || !codes || !scales || !biases || !aligned(x, 16) || !aligned(codes, 4) ||
      !aligned(scales, 2) || !aligned(biases, 2)) {
    set_error("am_q4_quantize: null or misaligned buffer (x needs 16-byte alignment)");
    return AM_ERR_INVALID;
  }
  return cuda_status(launch_quantize(x, dtype == AM_DTYPE_BF16, rows, dim, codes, scales, biases,
                                     static_cast<cudaStream_t>(stream)),
                     "am_q4_quantize");
}

int am_q4_dequantize(const uint32_t* codes, const void* scales, const void* biases,
                     int32_t scale_dtype, int64_t rows, int32_t dim, void* out, int32_t out_dtype,
                     void* stream) {
  clear_error();
  if (!valid_half_dtype(scale_dtype) || rows < 0 || dim <= 0 || dim % 64 ||
      !(valid_half_dtype(out_dtype) || out_dtype == AM_DTYPE_F32)) {
    set_error("am_q4_dequantize: bad dtype or dim");
    return AM_ERR_INVALID;
  }
  if (rows == 0) return AM_OK;
  if (!codes || !scales || !biases || !out) {
    set_error("am_q4_dequantize: null buffer");
    return AM_ERR_INVALID;
  }
  return cuda_status(launch_dequantize(codes, scales, biases, scale_dtype == AM_DTYPE_BF16, rows, dim,
                                       out, out_dtype, static_cast<cudaStream_t>(stream)),
                     "am_q4_dequantize");
}

int am_q4_append(const am_q4_cache* cache, const void* k, const void* v, int32_t dtype,
                 int32_t batch, int32_t n_new, int64_t k_stride_b, int64_t k_stride_h,
                 int64_t k_stride_l, int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_l,
                 const int32_t* positions, int32_t* status, void* stream) {
  clear_error();
  int rc = check_cache(cache, "am_q4_append");
  if (rc) return rc;
  if (dtype != cache->scale_dtype) {
    set_error("am_q4_append: input dtype must equal the cache's scale dtype");
    return AM_ERR_INVALID;
  }
  if (batch < 0 || n_new < 0) {
    set_error("am_q4_append: negative batch or n_new");
    return AM_ERR_INVALID;
  }
  if (batch == 0 || n_new == 0) return AM_OK;
  if (!k || !v || !positions || !aligned(k, 16) || !aligned(v, 16) ||
      ((k_stride_b | k_stride_h | k_stride_l | v_stride_b | v_stride_h | v_stride_l) % 8)) {
    set_error("am_q4_append: k/v must be 16-byte aligned with strides that are multiples of 8");
    return AM_ERR_INVALID;
  }
  if (cache->layout == AM_LAYOUT_CONTIGUOUS && batch > cache->batch) {
    set_error("am_q4_append: batch %d exceeds the cache's batch extent %d", batch, cache->batch);
    return AM_ERR_INVALID;
  }
  AppendParams p{};
  p.k = static_cast<const uint16_t*>(k);
  p.v = static_cast<const uint16_t*>(v);
  p.ksb = k_stride_b;
  p.ksh = k_stride_h;
  p.ksl = k_stride_l;
  p.vsb = v_stride_b;
  p.vsh = v_stride_h;
  p.vsl = v_stride_l;
  p.batch = batch;
  p.hkv = cache->n_kv_heads;
  p.n_new = n_new;
  p.k_dim = cache->k_dim;
  p.v_dim = cache->v_dim;
  p.positions = positions;
  p.kc = cache->k_codes;
  p.ks = static_cast<uint16_t*>(cache->k_scales);
  p.kb = static_cast<uint16_t*>(cache->k_biases);
  p.vc = cache->v_codes;
  p.vs = static_cast<uint16_t*>(cache->v_scales);
  p.vb = static_cast<uint16_t*>(cache->v_biases);
  p.layout = cache->layout;
  p.capacity = cache->capacity;
  p.block_tokens = cache->block_tokens;
  p.table_stride = cache->block_table_stride;
  p.table = cache->block_table;
  p.status = status;
  return cuda_status(launch_append(p, dtype == AM_DTYPE_BF16, static_cast<cudaStream_t>(stream)),
                     "am_q4_append");
}

size_t am_q4_decode_workspace_bytes(const am_q4_cache* cache, const am_attn_args* args) {
  if (cache == nullptr || args == nullptr || cache->n_kv_heads <= 0 || args->n_q_heads <= 0 ||
      args->batch < 0 || args->q_len < 0 || args->max_kv_len < 0)
    return 0;
  int row_groups, chunk, n_chunks, cluster;
  decode_geometry(cache, args, &row_groups, &chunk, &n_chunks, &cluster);
  if (n_chunks <= 1 || cluster) return 0;
  const size_t rows_total = static_cast<size_t>(args->n_q_heads) * args->q_len;
  return static_cast<size_t>(args->batch) * rows_total * n_chunks * (cache->v_dim + kPartialHead) *
         sizeof(float);
}

size_t am_q4_prefill_workspace_bytes(const am_q4_cache* cache, const am_attn_args* args) {
  if (cache == nullptr || args == nullptr || cache->n_kv_heads <= 0 || args->batch <= 0 ||
      args->q_len <= 0 || args->max_kv_len < 0 || cache->k_dim <= 0 || cache->v_dim <= 0)
    return 0;
  const PrefillPlanes pl = prefill_planes(cache, args);
  return pl.k_bytes + pl.v_bytes;
}

size_t am_q4_attention_workspace_bytes(const am_q4_cache* cache, const am_attn_args* args) {
  return routes_to_prefill(cache, args) ? am_q4_prefill_workspace_bytes(cache, args)
                                        : am_q4_decode_workspace_bytes(cache, args);
}

int am_q4_decode(const am_q4_cache* cache, const am_attn_args* a, void* workspace,
                 size_t workspace_bytes, void* stream) {
  clear_error();
  int rc = check_cache(cache, "am_q4_decode");
  if (rc) return rc;
  rc = check_args(cache, a, "am_q4_decode");
  if (rc) return rc;
  if (!decode_supported(cache->k_dim, cache->v_dim)) {
    set_error("am_q4_decode: no kernel for k_dim=%d v_dim=%d", cache->k_dim, cache->v_dim);
    return AM_ERR_UNSUPPORTED;
  }
  const int stage = decode_stage_tokens(cache->k_dim, cache->v_dim);
  if (cache->layout == AM_LAYOUT_PAGED &&
      (cache->block_tokens < stage || (cache->block_tokens & (cache->block_tokens - 1)))) {
    set_error("am_q4_decode: paged decode needs block_tokens to be a power of two >= %d (got %d)",
              stage, cache->block_tokens);
    return AM_ERR_UNSUPPORTED;
  }
  if (!aligned(cache->k_scales, 16) || !aligned(cache->k_biases, 16) ||
      !aligned(cache->v_scales, 16) || !aligned(cache->v_biases, 16)) {
    set_error("am_q4_decode: scales and biases must be 16-byte aligned (bulk copies)");
    return AM_ERR_INVALID;
  }
  const int n_rep = a->n_q_heads / cache->n_kv_heads;
  if (n_rep * a->q_len > 64) {
    set_error("am_q4_decode: n_rep * q_len = %d exceeds 64; use am_q4_prefill", n_rep * a->q_len);
    return AM_ERR_UNSUPPORTED;
  }
  if (a->batch == 0 || a->q_len == 0) return AM_OK;
  int row_groups, chunk, n_chunks, cluster;
  decode_geometry(cache, a, &row_groups, &chunk, &n_chunks, &cluster);
  const size_t need = am_q4_decode_workspace_bytes(cache, a);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 16))) {
    set_error("am_q4_decode: workspace of %zu bytes required (got %zu)", need, workspace_bytes);
    return AM_ERR_WORKSPACE;
  }
  DecodeParams p{};
  fill_params(p, cache, a);
  p.chunk = chunk;
  p.max_chunks = n_chunks;
  p.stage_tokens = decode_stage_tokens(cache->k_dim, cache->v_dim);
  p.ws = static_cast<float*>(workspace);
  p.cluster = cluster;
  if (decode_uses_tensor_maps(cache->k_dim, cache->v_dim)) {
    const int64_t rows = cache->layout == AM_LAYOUT_PAGED
                             ? cache->capacity * cache->n_kv_heads * cache->block_tokens
                             : static_cast<int64_t>(cache->batch) * cache->n_kv_heads * cache->capacity;
    if (rows <= 0 || rows > INT_MAX) {
      set_error("am_q4_decode: %lld code rows (sequences x KV heads x tokens) outside (0, 2^31)",
                static_cast<long long>(rows));
      return AM_ERR_UNSUPPORTED;
    }
    const int krow = cache->k_dim / 2, vrow = cache->v_dim / 2;
    const bool ksplit = krow == 96;
    if (!aligned(cache->k_codes, 16) || !aligned(cache->v_codes, 16) ||
        !encode_codes_map(&p.tmap_kc, cache->k_codes, rows, krow, ksplit ? 64 : krow, stage) ||
        (ksplit && !encode_codes_map(&p.tmap_kc2, cache->k_codes, rows, krow, 32, stage)) ||
        !encode_codes_map(&p.tmap_vc, cache->v_codes, rows, vrow, vrow, stage)) {
      set_error("am_q4_decode: cannot describe the K/V codes as tensor maps (16-byte aligned "
                "code arrays and a driver with cuTensorMapEncodeTiled are required)");
      return AM_ERR_CUDA;
    }
  }
  return cuda_status(launch_decode(p, a->batch, row_groups, cache->layout == AM_LAYOUT_PAGED,
                                   cache->scale_dtype == AM_DTYPE_BF16,
                                   static_cast<cudaStream_t>(stream)),
                     "am_q4_decode");
}

// One prefill call: the stage kernel over the keys in [key_lo, key_hi) and/or the attention
// kernel (parts), with the checks every prefill entry point shares.
static int prefill_call(const am_q4_cache* cache, const am_attn_args* a, void* workspace,
                        size_t workspace_bytes, void* stream, int key_lo, int key_hi, int parts,
                        const char* fn) {
  clear_error();
  int rc = check_cache(cache, fn);
  if (rc) return rc;
  rc = check_args(cache, a, fn);
  if (rc) return rc;
  if (!prefill_supported(cache->k_dim, cache->v_dim)) {
    set_error("%s: no kernel for k_dim=%d v_dim=%d", fn, cache->k_dim, cache->v_dim);
    return AM_ERR_UNSUPPORTED;
  }
  if (key_lo < 0 || key_hi < key_lo) {
    set_error("%s: key range [%d, %d) is not a range of key positions", fn, key_lo, key_hi);
    return AM_ERR_INVALID;
  }
  if (a->batch == 0 || a->q_len == 0) return AM_OK;
  const PrefillPlanes pl = prefill_planes(cache, a);
  const size_t need = pl.k_bytes + pl.v_bytes;
  if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 256)) {
    set_error("%s: a 256-byte aligned workspace of %zu bytes is required (got %zu)", fn, need,
              workspace_bytes);
    return AM_ERR_WORKSPACE;
  }
  if (pl.rows <= 0 || pl.rows > INT_MAX) {
    set_error("%s: %lld workspace rows (sequences x KV heads x keys) outside (0, 2^31)", fn,
              static_cast<long long>(pl.rows));
    return AM_ERR_UNSUPPORTED;
  }
  DecodeParams p{};
  fill_params(p, cache, a);
  p.kd = static_cast<uint16_t*>(workspace);
  p.vd = pl.v_bytes > 0 ? reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(workspace) + pl.k_bytes) : nullptr;
  p.nw = pl.nw;
  // The attention kernel reads rows up to its last key tile, which ends before key
  // max_kv_len + tile: rows of later keys are never read and not staged.  A range narrower
  // than the plane gets a grid of its own row blocks only (one more for the alignment of
  // the first).
  const int bn = prefill_key_tile(cache->k_dim, cache->v_dim);
  const int64_t hi_eff = std::min<int64_t>(key_hi, static_cast<int64_t>(a->max_kv_len) + bn);
  const int64_t range_rows = std::max<int64_t>(hi_eff - key_lo, 0);
  p.stage_lo = key_lo;
  p.stage_hi = static_cast<int32_t>(hi_eff);
  p.stage_blocks = range_rows + kStageRowsHost < pl.nw
                       ? static_cast<int32_t>((range_rows + kStageRowsHost - 1) / kStageRowsHost + 1)
                       : 0;
  if (!encode_codes_map(&p.tmap_kd, p.kd, pl.rows, cache->k_dim * 2, 128, bn) ||
      (pl.v_bytes > 0 && !encode_codes_map(&p.tmap_vd, p.vd, pl.rows, cache->v_dim * 2, 128, bn))) {
    set_error("%s: cannot describe the workspace as tensor maps (a driver with "
              "cuTensorMapEncodeTiled is required)", fn);
    return AM_ERR_CUDA;
  }
  return cuda_status(launch_prefill(p, a->batch, cache->layout == AM_LAYOUT_PAGED,
                                    cache->scale_dtype == AM_DTYPE_BF16, parts,
                                    static_cast<cudaStream_t>(stream)),
                     fn);
}

int am_q4_prefill(const am_q4_cache* cache, const am_attn_args* a, void* workspace,
                  size_t workspace_bytes, void* stream) {
  return prefill_call(cache, a, workspace, workspace_bytes, stream, 0, INT_MAX,
                      kPrefillStage | kPrefillAttend, "am_q4_prefill");
}

int am_q4_prefill_stage(const am_q4_cache* cache, const am_attn_args* a, int32_t key_lo,
                        int32_t key_hi, void* workspace, size_t workspace_bytes, void* stream) {
  return prefill_call(cache, a, workspace, workspace_bytes, stream, key_lo, key_hi, kPrefillStage,
                      "am_q4_prefill_stage");
}

int am_q4_prefill_attend(const am_q4_cache* cache, const am_attn_args* a, void* workspace,
                         size_t workspace_bytes, void* stream) {
  return prefill_call(cache, a, workspace, workspace_bytes, stream, 0, INT_MAX, kPrefillAttend,
                      "am_q4_prefill_attend");
}

int am_q4_attention(const am_q4_cache* cache, const am_attn_args* a, void* workspace,
                    size_t workspace_bytes, void* stream) {
  if (routes_to_prefill(cache, a)) return am_q4_prefill(cache, a, workspace, workspace_bytes, stream);
  return am_q4_decode(cache, a, workspace, workspace_bytes, stream);
}

static int blocks_copy(const am_q4_cache* pool, const int32_t* block_ids, const int32_t* tokens,
                       const int64_t* offsets, int32_t n_blocks, void* buffer, int32_t* status,
                       void* stream, bool to_buffer, const char* fn) {
  clear_error();
  if (pool == nullptr || pool->layout != AM_LAYOUT_PAGED) {
    set_error("%s: pool must describe a paged cache", fn);
    return AM_ERR_INVALID;
  }
  if (!pool->k_codes || !pool->k_scales || !pool->k_biases || !pool->v_codes || !pool->v_scales ||
      !pool->v_biases || !valid_half_dtype(pool->scale_dtype) || pool->n_kv_heads <= 0 ||
      pool->k_dim <= 0 || pool->v_dim <= 0 || pool->k_dim % 64 || pool->v_dim % 64 ||
      pool->block_tokens <= 0 || pool->capacity <= 0 || pool->capacity > INT32_MAX) {
    set_error("%s: incomplete pool description", fn);
    return AM_ERR_INVALID;
  }
  if (n_blocks < 0 || (n_blocks > 0 && (!block_ids || !tokens || !offsets || !buffer))) {
    set_error("%s: n_blocks >= 0 and block_ids, tokens, offsets, buffer required", fn);
    return AM_ERR_INVALID;
  }
  if (n_blocks == 0) return AM_OK;
  BlockCopyParams p{};
  p.pool[0] = const_cast<uint32_t*>(pool->k_codes);
  p.pool[1] = const_cast<void*>(pool->k_scales);
  p.pool[2] = const_cast<void*>(pool->k_biases);
  p.pool[3] = const_cast<uint32_t*>(pool->v_codes);
  p.pool[4] = const_cast<void*>(pool->v_scales);
  p.pool[5] = const_cast<void*>(pool->v_biases);
  p.row_bytes[0] = pool->k_dim / 2;
  p.row_bytes[1] = p.row_bytes[2] = pool->k_dim / 64 * 2;
  p.row_bytes[3] = pool->v_dim / 2;
  p.row_bytes[4] = p.row_bytes[5] = pool->v_dim / 64 * 2;
  p.hkv = pool->n_kv_heads;
  p.block_tokens = pool->block_tokens;
  p.num_blocks = static_cast<int32_t>(pool->capacity);
  p.block_ids = block_ids;
  p.tokens = tokens;
  p.offsets = offsets;
  p.buf = static_cast<uint8_t*>(buffer);
  p.to_buffer = to_buffer ? 1 : 0;
  p.status = status;
  return cuda_status(launch_blocks_copy(p, n_blocks, static_cast<cudaStream_t>(stream)), fn);
}

int am_q4_blocks_pack(const am_q4_cache* pool, const int32_t* block_ids, const int32_t* tokens,
                      const int64_t* offsets, int32_t n_blocks, void* buffer, int32_t* status,
                      void* stream) {
  return blocks_copy(pool, block_ids, tokens, offsets, n_blocks, buffer, status, stream, true,
                     "am_q4_blocks_pack");
}

int am_q4_blocks_unpack(const am_q4_cache* pool, const int32_t* block_ids, const int32_t* tokens,
                        const int64_t* offsets, int32_t n_blocks, const void* buffer,
                        int32_t* status, void* stream) {
  return blocks_copy(pool, block_ids, tokens, offsets, n_blocks, const_cast<void*>(buffer), status,
                     stream, false, "am_q4_blocks_unpack");
}

static int block_list_check(int32_t* free_ids, int32_t* free_top, int32_t num_blocks,
                            int32_t* table, int32_t table_stride, int32_t rows,
                            const int32_t* counts, const char* fn) {
  clear_error();
  if (!free_ids || !free_top || num_blocks <= 0 || rows < 0 || table_stride <= 0 ||
      (rows > 0 && (!table || !counts))) {
    set_error("%s: free list, table (stride > 0) and per-row counts required", fn);
    return AM_ERR_INVALID;
  }
  return AM_OK;
}

int am_block_reserve(int32_t* free_ids, int32_t* free_top, int32_t num_blocks, int32_t* table,
                     int32_t table_stride, int32_t rows, const int32_t* lengths,
                     const int32_t* add, int32_t block_tokens, int32_t* status, void* stream) {
  int rc = block_list_check(free_ids, free_top, num_blocks, table, table_stride, rows, add,
                            "am_block_reserve");
  if (rc) return rc;
  if (rows > 0 && (lengths == nullptr || block_tokens <= 0)) {
    set_error("am_block_reserve: lengths and block_tokens > 0 required");
    return AM_ERR_INVALID;
  }
  if (rows == 0) return AM_OK;
  BlockListParams p{};
  p.free_ids = free_ids;
  p.free_top = free_top;
  p.capacity = num_blocks;
  p.table = table;
  p.table_stride = table_stride;
  p.rows = rows;
  p.lengths = lengths;
  p.counts = add;
  p.block_tokens = block_tokens;
  p.status = status;
  return cuda_status(launch_block_reserve(p, static_cast<cudaStream_t>(stream)), "am_block_reserve");
}

int am_block_release(int32_t* free_ids, int32_t* free_top, int32_t num_blocks, int32_t* table,
                     int32_t table_stride, int32_t rows, const int32_t* keep_blocks,
                     int32_t* status, void* stream) {
  int rc = block_list_check(free_ids, free_top, num_blocks, table, table_stride, rows, keep_blocks,
                            "am_block_release");
  if (rc) return rc;
  if (rows == 0) return AM_OK;
  BlockListParams p{};
  p.free_ids = free_ids;
  p.free_top = free_top;
  p.capacity = num_blocks;
  p.table = table;
  p.table_stride = table_stride;
  p.rows = rows;
  p.counts = keep_blocks;
  p.status = status;
  return cuda_status(launch_block_release(p, static_cast<cudaStream_t>(stream)), "am_block_release");
}

}  // extern "C"
