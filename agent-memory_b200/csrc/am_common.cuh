// Shared device helpers and launch-parameter structs for the Q4 attention kernels.
// sm_100a only.  PTX used here: cp.async (LDGSTS), mma.sync m16n8k16, movmatrix,
// ex2.approx, and in the prefill kernel tcgen05.* / mbarrier.
#pragma once

#include <cuda.h>  // CUtensorMap (the type only; maps are encoded through the runtime's driver entry point)
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "am_q4.h"

namespace am {

constexpr int kGroup = 64;  // quantization group size along the head dimension

// ---------------------------------------------------------------- error reporting (host)
void set_error(const char* fmt, ...);
void clear_error();

// ---------------------------------------------------------------- 16-bit float loads
template <bool BF16>
__device__ __forceinline__ float h2f(uint16_t bits) {
  if constexpr (BF16) {
    return __uint_as_float(static_cast<uint32_t>(bits) << 16);
  } else {
    return __half2float(__ushort_as_half(bits));
  }
}

template <bool BF16>
__device__ __forceinline__ uint16_t f2h(float v) {
  if constexpr (BF16) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  } else {
    return __half_as_ushort(__float2half_rn(v));
  }
}

__device__ __forceinline__ float h2f_rt(uint16_t bits, bool bf16) {
  return bf16 ? h2f<true>(bits) : h2f<false>(bits);
}

// Store one fp32 value as dtype (AM_DTYPE_F16 / BF16 / F32).
__device__ __forceinline__ void store_out(void* base, int64_t idx, float v, int dtype) {
  if (dtype == AM_DTYPE_F32) {
    static_cast<float*>(base)[idx] = v;
  } else if (dtype == AM_DTYPE_BF16) {
    static_cast<uint16_t*>(base)[idx] = f2h<true>(v);
  } else {
    static_cast<uint16_t*>(base)[idx] = f2h<false>(v);
  }
}

// ---------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst)), "l"(src));
}

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(dst)), "l"(src));
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// D += A(16x16, f16, row) * B(16x8, f16, col), fp32 accumulators.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D += A(16x16, bf16, row) * B(16x8, bf16, col), fp32 accumulators.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four 8x8 b16 matrices from shared memory, transposed: lane L supplies the row address
// (16 bytes) of row L % 8 of matrix L / 8; lane (g, t) receives in r_k the b16 elements
// (row 2t, column g) [low half] and (row 2t + 1, column g) [high half] of matrix k.
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Transpose an 8x8 matrix of 16-bit values held in mma fragment layout across the warp.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ---------------------------------------------------------------- mbarrier / bulk copy
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes)
               : "memory");
}

// 1-D bulk copy global -> shared (TMA engine, no multicast); completes `bytes` on `bar`.
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// 2-D tiled TMA load (no multicast) of the box at (x, y) of `map` into shared memory,
// completing on mbarrier `bar`.  `map` must live in parameter, constant or global memory.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Shared-memory address of byte `byte` of row `row` in a tile of ROWB-byte rows written by a
// TMA load with the matching swizzle (ROWB = 32, 64, 128 <-> CU_TENSOR_MAP_SWIZZLE_32B, 64B,
// 128B): the 16-byte chunk index is XORed with address bits 7.. of the row start, so rows
// that share a chunk column land in different banks.  `base` is aligned to the pattern
// period (256, 512 or 1024 bytes).
template <int ROWB>
__device__ __forceinline__ uint32_t swz_addr(uint32_t base, int row, int byte) {
  static_assert(ROWB == 32 || ROWB == 64 || ROWB == 128, "swizzled rows are 32, 64 or 128 bytes");
  constexpr int SH = ROWB == 128 ? 0 : (ROWB == 64 ? 1 : 2);  // rows per 128-byte line: 1, 2, 4
  constexpr int MASK = ROWB == 128 ? 7 : (ROWB == 64 ? 3 : 1);
  const int chunk = (byte >> 4) ^ ((row >> SH) & MASK);
  return base + row * ROWB + (chunk << 4) + (byte & 15);
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}

// Default limit of a kernel's bounded waits (DecodeParams::wait_ns): 2 s.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Wait for phase `parity` of an mbarrier; gives up after `limit_ns` (returns false).  Each
// try_wait may suspend the warp for up to 0.5 ms (woken early when the phase completes), so
// a waiting warp yields its issue slots instead of spinning.  limit_ns == 0 gives up at once,
// as a wait whose phase never completes would after its limit: tests use it to drive a
// kernel's timeout path (flag, drain the copies in flight, release, return) without
// waiting for anything.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  uint64_t limit_ns = kWaitLimitNs) {
  constexpr uint32_t kSuspendNs = 500000;
  if (limit_ns == 0) return false;
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    uint32_t done;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        "selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(kSuspendNs)
        : "memory");
    if (done) return true;
    if (it == 0) {
      t0 = globaltimer_ns();
    } else if (globaltimer_ns() - t0 > limit_ns) {
      return false;
    }
  }
}

__device__ __forceinline__ void flag_status(int32_t* status, int bits) {
  if (status != nullptr) atomicOr(status, bits);
}

// Programmatic dependent launch.  griddep_wait() returns once every grid this one depends
// on has completed and its writes are visible (immediately when the grid was launched
// without the programmatic-serialization attribute); griddep_launch_dependents() lets the
// next grid in the stream start its prologue early.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

// Thread-block cluster primitives: a full cluster barrier (every thread of every CTA of the
// cluster; writes before it are visible to reads after it across the cluster), the
// distributed-shared-memory address of a peer CTA's copy of a local shared address, and
// a 32-bit load through that address.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];\n" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Final softmax normalisation of one query row from its running max m and sum l (log2
// units), with an optional attention sink s2 (log2 units): returns the factor that turns
// the unnormalised output O into O * w / den, i.e. w / den, so that
// out = O * factor.  Without a sink: 1 / l.  With one: the sink joins max and sum.
__device__ __forceinline__ float softmax_out_factor(float m, float l, bool has_sink, float s2) {
  if (!has_sink) return l > 0.0f ? __fdividef(1.0f, l) : 0.0f;
  const float mm = fmaxf(m, s2);
  const float w = m == -INFINITY ? 0.0f : exp2f(m - mm);
  const float den = fmaf(l, w, exp2f(s2 - mm));
  return den > 0.0f ? __fdividef(w, den) : 0.0f;
}

// Split-KV partial record of one query row and chunk: m, l, two pad words (so O starts
// 16-byte aligned), then O[DV].
constexpr int kPartialHead = 4;

// ---------------------------------------------------------------- launch parameters

// Whole-block copies between the pool and a packed buffer (am_blocks.cu).  Sections:
// 0 K weights, 1 K scales, 2 K biases, 3 V weights, 4 V scales, 5 V biases.
struct BlockCopyParams {
  void* pool[6];
  int64_t row_bytes[6];
  int32_t hkv, block_tokens, num_blocks;
  const int32_t* block_ids;
  const int32_t* tokens;
  const int64_t* offsets;  // [n_blocks][6] byte offsets into buf
  uint8_t* buf;
  int32_t to_buffer;
  int32_t* status;
};

// Device free list (am_blocks.cu).  counts = tokens to add (reserve) or blocks to keep
// (release) per row.
struct BlockListParams {
  int32_t* free_ids;
  int32_t* free_top;
  int32_t capacity;
  int32_t* table;
  int32_t table_stride;
  int32_t rows;
  const int32_t* lengths;
  const int32_t* counts;
  int32_t block_tokens;
  int32_t* status;
};

// Quantize-on-append / plain quantize.  Rows are (b, h, l) triples of the source tensors.
struct AppendParams {
  const uint16_t* k;
  const uint16_t* v;
  int64_t ksb, ksh, ksl;  // element strides of the new K rows
  int64_t vsb, vsh, vsl;
  int32_t batch, hkv, n_new;
  int32_t k_dim, v_dim;
  const int32_t* positions;  // [batch] first destination position
  // destination cache
  uint32_t* kc;
  uint16_t* ks;
  uint16_t* kb;
  uint32_t* vc;
  uint16_t* vs;
  uint16_t* vb;
  int32_t layout;
  int64_t capacity;  // contiguous rows per (b, h) or paged num_blocks
  int32_t block_tokens;
  int32_t table_stride;
  const int32_t* table;
  int32_t* status;
};

// Split-KV decode attention.
struct DecodeParams {
  const uint32_t* kc;
  const uint16_t* ks;
  const uint16_t* kb;
  const uint32_t* vc;
  const uint16_t* vs;
  const uint16_t* vb;
  int64_t capacity;
  const int32_t* table;
  int32_t table_stride;
  int32_t block_tokens;
  int32_t bt_shift;  // log2(block_tokens) for paged decode
  int32_t hkv;
  int32_t k_dim;
  int32_t v_dim;
  int32_t hq;
  int32_t q_len;
  int32_t n_rep;
  int32_t rows_per_head;  // n_rep * q_len
  int32_t stage_tokens;   // decode pipeline stage (tokens); visible ranges align to it
  int32_t q_bf16;
  const uint16_t* q;
  int64_t qsb, qsh, qsl;
  void* out;
  int32_t out_dtype;
  int64_t osb, osh, osl;
  float scale_log2;  // softmax scale * log2(e)
  const int32_t* kv_len;
  const int32_t* kv_start;
  int32_t causal;
  int32_t window;
  int32_t mask_kind;
  int32_t mask_dtype;
  const void* mask;
  int64_t msb, msh, msl, msn;
  int32_t* status;
  int32_t chunk;       // tokens per split (multiple of 64)
  int32_t max_chunks;  // grid.x
  float* ws;           // partials [batch][hq*q_len][max_chunks][kPartialHead + v_dim]
  const float* sinks;  // [hq] sink logits (scaled-score units) or nullptr
  uint64_t wait_ns;    // limit of the kernels' bounded waits (kWaitLimitNs unless a test lowers it)
  int32_t cluster;     // 1: the max_chunks CTAs of a column are one thread-block cluster and
                       // merge their partials through distributed shared memory (no ws)
  // Decode kernels whose code rows are 32, 64 or 128 bytes load K and V codes through these
  // 2-D tensor maps ([rows, row bytes], box = one stage, swizzled to the row size).
  // (Dk = 192: tmap_kc holds bytes 0..63 of each 96-byte K row, tmap_kc2 bytes 64..95)
  alignas(64) CUtensorMap tmap_kc;
  alignas(64) CUtensorMap tmap_vc;
  alignas(64) CUtensorMap tmap_kc2;
  // Prefill: fp16 rows of the keys and values the query block can see, dequantized by the
  // stage kernel into the caller's workspace ([batch][hkv][nw][k_dim] and [..][v_dim]), and
  // the 2-D tensor maps the attention kernel loads them through ([rows, row bytes], box =
  // 128 bytes x one key tile, 128-byte swizzle).
  uint16_t* kd;
  uint16_t* vd;
  int32_t nw;  // rows per (sequence, KV head) plane
  // The stage kernel writes only the rows of keys in [stage_lo, stage_hi) (absolute key
  // positions); am_q4_prefill stages every row, am_q4_prefill_stage a range of them.
  int32_t stage_lo;
  int32_t stage_hi;
  // Row blocks of the stage grid (grid.x): 0 = every block of the plane; otherwise the grid
  // covers only the blocks from the one holding key stage_lo on.
  int32_t stage_blocks;
  // Prefill kernels that dequantize V tiles themselves read the cache directly: block-pool
  // layout (table, block_tokens) or contiguous rows, and the scale / bias type.
  int32_t paged;
  int32_t scale_bf16;
  alignas(64) CUtensorMap tmap_kd;
  alignas(64) CUtensorMap tmap_vd;
};

// Visible key range of a sequence for the structured mask: keys outside [lo, hi) are
// excluded for every query row.  lo is rounded down to a multiple of `align` (the decode
// stage size, a power of two).
__device__ __forceinline__ void visible_range(int n, int st, int q_len, int window, bool dense_mask,
                                              int align, int& lo, int& hi) {
  hi = n;
  if (dense_mask) {
    lo = 0;
  } else {
    lo = st;
    if (window > 0) lo = max(lo, n - q_len - window + 1);
    lo = max(lo, 0);
  }
  lo &= ~(align - 1);  // pipeline stages start on stage boundaries
}

}  // namespace am
