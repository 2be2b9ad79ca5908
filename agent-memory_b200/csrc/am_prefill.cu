// Chunked-prefill attention over a Q4 cache on 5th-generation tensor cores (tcgen05), in two
// launches.
//
// 1. prefill_stage_kernel dequantizes, once per call, every key and value a query block can
//    see into fp16 rows of a caller-provided workspace: one plane of `nw` rows per (sequence,
//    KV head), row r holding key lo_b + r, where [lo_b, kv_len) is the union of the block's
//    visible ranges (left padding and sliding window applied; a dense mask sees every key).
//    Rows outside that range, past the end of the cache, or behind a bad block id are
//    zeros, so every row a tile can reach is finite.  code * scale + bias is formed in fp32
//    and rounded once to fp16 (saturating at +-65504).  HBM-bound: reads Dk/2 + Dk/16 +
//    Dv/2 + Dv/16 bytes and writes 2 (Dk + Dv) bytes per (key, KV head) -- 2 Dk for MLA's
//    192 / 128, whose V tiles the attention kernel dequantizes itself (HBM writes bound
//    the stage, and at that shape they are 31% of the layer).
//
// 2. The attention kernel streams the fp16 planes.  Query rows are (token, GQA head) pairs,
//    token-major, so each K/V tile feeds the n_rep heads that share its KV head.  Two
//    variants, chosen by head dims:
//    * prefill2_kernel (Dk, Dv <= 128): one CTA = two 128-row query tiles of one KV head of
//      one sequence, 320 threads.  One thread of warp 8 streams 128-key K and V tiles into
//      NS-stage shared-memory rings with 2-D tensor-map TMA loads (128-byte swizzle, no
//      multicast); one thread of warp 9 issues every tcgen05.mma (kind::f16, M = 128,
//      N = 128, 16-deep steps): S = Q . K^T into TMEM S[qt], then O[qt] += P . V with P read
//      from TMEM, alternating the tiles (S0_i, PV1_{i-1}, S1_i, PV0_i) so the tensor core
//      works on one tile while the softmax warps of the other run; softmax warps 0-7, four
//      per tile, one thread per query row and all 128 key columns of a tile.
//    * prefill_kernel (MLA 192/128 and Gemma-3 256/256, whose two tiles do not fit in TMEM):
//      one CTA = one 128-row query tile, 320 threads; BN-key tiles (128, or 64 for Dk + Dv >
//      384); 8 softmax warps, two per TMEM lane quarter, each owning BN / 2 key columns of
//      every tile and exchanging row maxima with its partner through shared memory; the
//      tensor core computes S_j while the softmax warps work on tile j-1.  For MLA, four
//      more warps (448 threads) fill the V ring from the Q4 cache: one thread per key keeps
//      its code words, scales and biases for three tiles in registers and writes the
//      swizzled fp16 rows with f16x2 arithmetic (rows with a group beyond fp16's range take
//      an out-of-line fp32 path that saturates); the TMA thread then streams K only.
//    Both: tcgen05.ld of the scores, fp32 online softmax, P as fp16 pairs stored back over
//    the S columns (tcgen05.st); O rows rescaled in TMEM only when the running max moves by
//    more than 2^8.  The two-tile kernel computes P against the running max in one read of
//    the scores and takes the row max only when a tile's sum leaves the fp16 range of P (or
//    for a row's first tile); the one-tile kernel takes the row max every tile and runs a
//    fixed share of its exponentials as a polynomial on the FMA pipe (ex2_fma below).
//    mbarriers chain the stages: TMA completions (K/V full), MMA commits (S full, O full,
//    K/V empty) and the softmax threads' arrivals (P full).  TMEM: 512 columns, one CTA per
//    SM.  Operands are fp16: queries (fp16 or bf16) are rescaled per row by a power of two
//    so their conversion is exact.  Every wait is bounded (DecodeParams::wait_ns, 2 s); on
//    timeout the kernel flags AM_STATUS_TIMEOUT, stops issuing work, waits (bounded) for
//    its TMA loads and MMAs in flight, frees its TMEM and returns.
//
// The attention grid is launched with programmatic stream serialization: its prologue (TMEM
// allocation, barriers, the query tile) overlaps the end of the stage kernel, and the TMA
// thread waits in griddepcontrol.wait before it reads the workspace.
//
// Reference semantics: the compiled quantized SDPA (mlx_fused_attention.py:69-139) as used
// by chunked prefill (batch_engine.py:339-456): the chunk's own K/V are already in the Q4
// cache (quantize-on-append runs first, mlx_quantized_extensions.py:273-298) and query l
// of the chunk sits at position kv_len - q_len + l.
#include "am_common.cuh"
#include "am_internal.h"

namespace am {

namespace tc {

// Shared-memory matrix descriptor (sm_100): 128-byte swizzle, start / leading / stride byte
// offsets in 16-byte units.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;  // 128-byte swizzle
  return d;
}

// kind::f16 instruction descriptor: fp16 A/B, fp32 D, A K-major, B K- or MN-major.
__host__ __device__ constexpr uint32_t idesc(int m, int n, bool b_mn_major) {
  return (1u << 4) | (b_mn_major ? (1u << 16) : 0u) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

// D (TMEM) [+]= A (shared-memory descriptor) x B (shared-memory descriptor).
__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t id,
                                    uint32_t accum) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(id), "r"(accum));
}

// D (TMEM) [+]= A (TMEM: M rows in lanes, K fp16 elements packed two per 32-bit column)
// x B (shared-memory descriptor).
__device__ __forceinline__ void mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t id,
                                       uint32_t accum) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(id), "r"(accum));
}

// Arrive on `bar` once every tcgen05 operation this thread issued before has completed.
__device__ __forceinline__ void commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
      bar)
               : "memory");
}

__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}

#define AM_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), \
                 "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])

// Warp loads 32 lanes x 32 consecutive fp32 columns of TMEM (thread i <- lane base+i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : AM_R8(0), AM_R8(8), AM_R8(16), AM_R8(24)
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Warp loads 32 lanes x 64 consecutive fp32 columns of TMEM in one instruction.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {"
      "%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n"
      : AM_R8(0), AM_R8(8), AM_R8(16), AM_R8(24), AM_R8(32), AM_R8(40), AM_R8(48), AM_R8(56)
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}
#undef AM_R8

// Warp loads 32 lanes x 16 consecutive fp32 columns of TMEM.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// The x64 load without its wait (tcgen05.wait::ld separately, before the values are used).
__device__ __forceinline__ void tmem_ld64_nowait(uint32_t taddr, float (&v)[64]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
#define AM_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), \
                 "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {"
      "%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n"
      : AM_R8(0), AM_R8(8), AM_R8(16), AM_R8(24), AM_R8(32), AM_R8(40), AM_R8(48), AM_R8(56)
      : "r"(taddr));
#undef AM_R8
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float (&v)[N]) {
  static_assert(N == 16 || N == 32 || N == 64, "16, 32 or 64 columns");
  if constexpr (N == 64) {
    tmem_ld64(taddr, v);
  } else if constexpr (N == 32) {
    tmem_ld32(taddr, v);
  } else {
    tmem_ld16(taddr, v);
  }
}

// Warp stores 32 lanes x 32 consecutive 32-bit columns of TMEM (thread i -> lane base+i).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
      "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
      "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}

// Warp stores 32 lanes x 16 consecutive 32-bit columns of TMEM.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};\n" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}

template <int N>
__device__ __forceinline__ void tmem_st(uint32_t taddr, const uint32_t (&v)[N]) {
  static_assert(N == 16 || N == 32, "16 or 32 columns");
  if constexpr (N == 32) {
    tmem_st32(taddr, v);
  } else {
    tmem_st16(taddr, v);
  }
}

// Warp stores 32 lanes x N fp32 columns (N = 16 or 32).
template <int N>
__device__ __forceinline__ void tmem_stf(uint32_t taddr, const float (&v)[N]) {
  uint32_t u[N];
#pragma unroll
  for (int i = 0; i < N; ++i) u[i] = __float_as_uint(v[i]);
  tmem_st<N>(taddr, u);
}

}  // namespace tc

// 2^x on the FMA pipe for x in [-125, 8] (Cody-Waite range reduction, W. J. Cody and
// W. Waite, "Software Manual for the Elementary Functions", Prentice-Hall 1980, and a cubic
// minimax polynomial): x = j + f with j = rint(x) taken from the low mantissa bits of
// x + 1.5 * 2^23 and f in [-0.5, 0.5]; 2^f ~= c0 + f (c1 + f (c2 + f c3)); the result's
// exponent is raised by j with one integer add.  The coefficients minimise the relative
// error on [-0.5, 0.5] (Remez exchange, derived for this kernel): max relative error
// 7.5e-5, below the fp16 rounding of P (2^-11).
__device__ __forceinline__ float ex2_fma(float x) {
  x = fmaxf(x, -125.0f);
  const float t = x + 12582912.0f;         // 1.5 * 2^23: rounds x to an integer in t's mantissa
  const float f = x - (t - 12582912.0f);   // in [-0.5, 0.5]
  float p = fmaf(f, 0.0551716685295105f, 0.2426111251115799f);
  p = fmaf(f, p, 0.6932609677314758f);
  p = fmaf(f, p, 0.9999280571937561f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// The same on a pair of values with the packed fp32x2 FMA pipe operations of sm_100 (two
// lanes per instruction for the range reduction and the polynomial).
__device__ __forceinline__ float2 ex2_fma2(float2 x) {
  // clamped to [-125, 64]: the exponent add below stays inside the float's exponent range
  // (a larger argument, possible against a running max that has fallen behind, must give a
  // large value, not a wrapped one)
  x.x = fminf(fmaxf(x.x, -125.0f), 64.0f);
  x.y = fminf(fmaxf(x.y, -125.0f), 64.0f);
  const float2 big = make_float2(12582912.0f, 12582912.0f);
  const float2 t = __fadd2_rn(x, big);
  const float2 j = __fadd2_rn(t, make_float2(-12582912.0f, -12582912.0f));
  const float2 f = __ffma2_rn(j, make_float2(-1.0f, -1.0f), x);  // in [-0.5, 0.5]
  float2 q = __ffma2_rn(f, make_float2(0.0551716685295105f, 0.0551716685295105f),
                        make_float2(0.2426111251115799f, 0.2426111251115799f));
  q = __ffma2_rn(f, q, make_float2(0.6932609677314758f, 0.6932609677314758f));
  q = __ffma2_rn(f, q, make_float2(0.9999280571937561f, 0.9999280571937561f));
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

// Three-input maximum (one instruction on sm_100).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Exponentials of softmax element pairs (2c, 2c+1): with kFmaExpEvery > 0, pairs with
// c % kFmaExpEvery == kFmaExpEvery - 1 go through the FMA-pipe polynomial, the rest through
// the MUFU unit; 0 keeps every exponential on the MUFU unit.  One-tile kernel: a quarter on
// the FMA pipe.  Two-tile kernel (one thread per query row, 128 exponentials per tile): a
// quarter measured best while every tile also took a max pass (655 TFLOP/s against 645 with
// none and 632 with half); with the one-pass softmax all on the MUFU unit measures best (700
// against 686 with a quarter and 679 with a third).
constexpr int kFmaExpEvery = 4;
constexpr int kTile2FmaExpEvery = 0;

// Lazy rescaling: a row's running max is raised only when a tile's max exceeds it by more
// than 2^8 (log2 units), so P <= 256 (exact range for the fp16 P operand) and the O
// accumulator in TMEM is rescaled rarely.
constexpr float kPrefillRescaleSlack = 8.0f;

// ---------------------------------------------------------------- visible range
// Keys a query block of sequence b can see, over all its queries: [lo, hi).
__device__ __forceinline__ void prefill_block_range(const DecodeParams& p, int b, int& lo, int& hi) {
  const int n = max(p.kv_len[b], 0);
  hi = n;
  lo = 0;
  if (p.mask_kind == AM_MASK_NONE) {
    lo = p.kv_start != nullptr ? max(p.kv_start[b], 0) : 0;
    if (p.window > 0) lo = max(lo, n - p.q_len - p.window + 1);
  }
  lo = min(lo, hi);
}

// ---------------------------------------------------------------- query tiles
// A thread stages CH 16-byte chunks (8 elements each) of a query row: all loads issued at
// once (one memory latency per CTA prologue rather than one per chunk), the row's max |q|
// taken from the registers, then each chunk converted to fp16 times a power of two and
// stored into the 128-byte-swizzled query tile.
template <int CH>
__device__ __forceinline__ void q_chunks_load(const uint16_t* src, bool ok, uint4 (&raw)[CH]) {
  if (ok) {
#pragma unroll
    for (int c = 0; c < CH; ++c) raw[c] = *reinterpret_cast<const uint4*>(src + c * 8);
  } else {
#pragma unroll
    for (int c = 0; c < CH; ++c) raw[c] = make_uint4(0, 0, 0, 0);
  }
}

template <int CH>
__device__ __forceinline__ float q_chunks_amax(const uint4 (&raw)[CH], bool bf16) {
  float amax = 0.0f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const uint32_t u[4] = {raw[c].x, raw[c].y, raw[c].z, raw[c].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      amax = fmaxf(amax, fabsf(h2f_rt(u[i] & 0xffffu, bf16)));
      amax = fmaxf(amax, fabsf(h2f_rt(u[i] >> 16, bf16)));
    }
  }
  return amax;
}

// The power of two that puts a row's max |q| just below 2^15 (1 for an empty or non-finite
// row), negated for a negative softmax scale so the factor back to scaled log2 scores is
// always positive.
__device__ __forceinline__ float q_row_prescale(float amax, float scale_log2) {
  float pw = 1.0f;
  if (amax > 0.0f && isfinite(amax)) {
    int e;
    frexpf(amax, &e);
    pw = ldexpf(1.0f, 15 - e);
  }
  return scale_log2 < 0.0f ? -pw : pw;
}

// Chunks c0 .. c0 + CH - 1 of row r into a query tile of 64-element slabs (QSLAB bytes).
template <int CH>
__device__ __forceinline__ void q_chunks_store(uint8_t* tile, int qslab, const uint4 (&raw)[CH], float pw,
                                               bool bf16, int r, int c0) {
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const uint32_t u[4] = {raw[c].x, raw[c].y, raw[c].z, raw[c].w};
    uint32_t o4[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o4[i] = pack_half2(h2f_rt(u[i] & 0xffffu, bf16) * pw, h2f_rt(u[i] >> 16, bf16) * pw);
    const int cc = c0 + c;
    const uint32_t off = (cc / 8) * qslab + r * 128 + (cc % 8) * 16;
    *reinterpret_cast<uint4*>(tile + (off ^ (((off >> 7) & 7u) << 4))) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
  }
}

// ---------------------------------------------------------------- stage kernel
// grid (ceil(nw / kStageRows), Hkv, batch), 256 threads.  A block converts kStageRows rows of
// plane (b, h); the work items are 16-byte chunks of code words (32 elements each, K chunks
// then V chunks of a row), and each thread issues the loads of all its items (codes, scale,
// bias) before converting any, so enough bytes are in flight to stream at HBM speed.
constexpr int kStageRows = kStageRowsHost;

// One 32-byte store of 8 words (p 32-byte aligned).
__device__ __forceinline__ void st_global_v8(void* p, const uint32_t (&v)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

template <int DK, int DV, bool SBF16, bool PAGED, bool KONLY>
__global__ void __launch_bounds__(256) prefill_stage_kernel(const __grid_constant__ DecodeParams p) {
  griddep_launch_dependents();
  // (KONLY: the attention kernel dequantizes V itself; only the K plane is written)
  constexpr int CK = DK / 32, CV = KONLY ? 0 : DV / 32, CPR = CK + CV;  // chunks per row
  constexpr int ITEMS = (kStageRows * CPR + 255) / 256;
  constexpr int NGK = DK / 64, NGV = DV / 64;
  const int h = blockIdx.y, b = blockIdx.z;
  int lo, hi;
  prefill_block_range(p, b, lo, hi);
  // a grid sized for a key range starts at the row block holding key stage_lo
  const int r_base =
      p.stage_blocks > 0 ? (min(max(p.stage_lo - lo, 0), p.nw) & ~(kStageRows - 1)) : 0;
  const int r0 = r_base + blockIdx.x * kStageRows;
  if (hi - lo > p.nw) {  // kv_len beyond the max_kv_len the workspace was sized for
    if (blockIdx.x == 0 && h == 0 && threadIdx.x == 0) flag_status(p.status, AM_STATUS_BAD_POSITION);
    hi = lo + p.nw;
  }
  // rows of keys outside [stage_lo, stage_hi) belong to another stage call: left untouched
  if (lo + r0 >= p.stage_hi || lo + r0 + kStageRows <= p.stage_lo) return;
  uint4 code[ITEMS];
  uint16_t sc[ITEMS], bi[ITEMS];
  bool live[ITEMS];
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) {
    const int item = threadIdx.x + 256 * k;
    const int r = r0 + item / CPR, c = item % CPR;
    const int t = lo + r;
    live[k] = false;
    code[k] = make_uint4(0, 0, 0, 0);
    sc[k] = bi[k] = 0;
    if (item < kStageRows * CPR && r < p.nw && t < hi && t >= p.stage_lo && t < p.stage_hi) {
      int64_t row = -1;
      if constexpr (PAGED) {
        const int blk_i = t / p.block_tokens;
        const int32_t blk = blk_i < p.table_stride ? p.table[(int64_t)b * p.table_stride + blk_i] : -1;
        if (blk < 0 || blk >= p.capacity) {
          flag_status(p.status, AM_STATUS_BAD_BLOCK);
        } else {
          row = ((int64_t)blk * p.hkv + h) * p.block_tokens + t % p.block_tokens;
        }
      } else {
        if (t < p.capacity) {
          row = ((int64_t)b * p.hkv + h) * p.capacity + t;
        } else {
          flag_status(p.status, AM_STATUS_BAD_POSITION);
        }
      }
      if (row >= 0) {
        live[k] = true;
        if (c < CK) {
          code[k] = __ldg(reinterpret_cast<const uint4*>(p.kc + row * (DK / 8)) + c);
          sc[k] = __ldg(p.ks + row * NGK + c / 2);
          bi[k] = __ldg(p.kb + row * NGK + c / 2);
        } else {
          code[k] = __ldg(reinterpret_cast<const uint4*>(p.vc + row * (DV / 8)) + (c - CK));
          sc[k] = __ldg(p.vs + row * NGV + (c - CK) / 2);
          bi[k] = __ldg(p.vb + row * NGV + (c - CK) / 2);
        }
      }
    }
  }
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) {
    const int item = threadIdx.x + 256 * k;
    const int r = r0 + item / CPR, c = item % CPR;
    if (item >= kStageRows * CPR || r >= p.nw || lo + r < p.stage_lo || lo + r >= p.stage_hi) continue;
    const int64_t plane_row = ((int64_t)b * p.hkv + h) * p.nw + r;
    uint16_t* dst = c < CK ? p.kd + plane_row * DK + c * 32 : p.vd + plane_row * DV + (c - CK) * 32;
    const float s = h2f<SBF16>(sc[k]), bias = h2f<SBF16>(bi[k]);
    const uint32_t w[4] = {code[k].x, code[k].y, code[k].z, code[k].w};
    // the chunk's 64 output bytes as two 32-byte stores: each one writes whole sectors
    // (dst is 64-byte aligned: planes start on 256 bytes, rows and chunks are 64-byte
    // multiples)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t o[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
      if (live[k]) {
#pragma unroll
        for (int qq = 0; qq < 2; ++qq) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            // a code OR-ed into the mantissa of 2^23 is exactly 2^23 + code (no int->float
            // conversion on the XU pipe)
            const uint32_t wq = w[2 * half + qq];
            const float c0 = __int_as_float(0x4B000000 | ((wq >> (8 * e)) & 15u)) - 8388608.0f;
            const float c1 = __int_as_float(0x4B000000 | ((wq >> (8 * e + 4)) & 15u)) - 8388608.0f;
            float x0 = fmaf(c0, s, bias);
            float x1 = fmaf(c1, s, bias);
            x0 = fminf(fmaxf(x0, -65504.0f), 65504.0f);
            x1 = fminf(fmaxf(x1, -65504.0f), 65504.0f);
            o[4 * qq + e] = pack_half2(x0, x1);
          }
        }
      }
      st_global_v8(dst + 16 * half, o);
    }
  }
}

// ---------------------------------------------------------------- in-kernel V dequantization
// The one-tile attention kernel (Dk or Dv > 128) takes K from the stage kernel's fp16 plane
// but converts its V tiles itself, straight from the Q4 cache: the stage then writes half
// the bytes (HBM writes bound it), and each V tile crosses from L2 as Q4 (3.5x fewer bytes).
// One code word (8 elements) becomes one 16-byte operand chunk of fp16 pairs in the order
// (e0, e4), (e1, e5), (e2, e6), (e3, e7): a nibble pair 16 bits apart, OR-ed into the
// mantissas of two copies of 1024.0, is exactly (1024 + code) in each half, so one LOP3 and
// one subtraction give two exact codes, and fma.rn.f16x2 forms code * scale + bias with a
// single rounding.  O's columns then hold the elements of each 8-element chunk in that
// order, and the epilogue reads them back in element order.
__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint4 q4_word_f16(uint32_t w, uint32_t s2, uint32_t b2) {
  constexpr uint32_t kLo = 0x000F000Fu, k1024 = 0x64006400u;
  const uint32_t x0 = (w & kLo) | k1024, x1 = ((w >> 4) & kLo) | k1024;
  const uint32_t x2 = ((w >> 8) & kLo) | k1024, x3 = ((w >> 12) & kLo) | k1024;
  return make_uint4(hfma2_u32(hsub2_u32(x0, k1024), s2, b2), hfma2_u32(hsub2_u32(x1, k1024), s2, b2),
                    hfma2_u32(hsub2_u32(x2, k1024), s2, b2), hfma2_u32(hsub2_u32(x3, k1024), s2, b2));
}

// The same word the stage kernel's way: code * scale + bias in fp32, saturated at +-65504,
// rounded once to fp16 (for groups whose values leave the fp16 range).
__device__ __forceinline__ uint4 q4_word_f32(uint32_t w, float s, float b) {
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float c0 = __int_as_float(0x4B000000 | ((w >> (4 * e)) & 15u)) - 8388608.0f;
    const float c1 = __int_as_float(0x4B000000 | ((w >> (4 * e + 16)) & 15u)) - 8388608.0f;
    o[e] = pack_half2(fminf(fmaxf(fmaf(c0, s, b), -65504.0f), 65504.0f),
                      fminf(fmaxf(fmaf(c1, s, b), -65504.0f), 65504.0f));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// A group's scale and bias as floats from (scale | bias << 16).
__device__ __forceinline__ void q4_group_f32(uint32_t sb, bool sbf16, float& s, float& b) {
  s = sbf16 ? __uint_as_float(sb << 16) : h2f<false>(static_cast<uint16_t>(sb & 0xffffu));
  b = sbf16 ? __uint_as_float(sb & 0xffff0000u) : h2f<false>(static_cast<uint16_t>(sb >> 16));
}

// code * scale + bias is monotonic in the code, so codes 0 and 15 bound a group's values.
template <int NG>
__device__ __forceinline__ bool q4_groups_in_f16_range(const uint32_t (&sb)[NG], bool sbf16) {
  bool ok = true;
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    float s, b;
    q4_group_f32(sb[g], sbf16, s, b);
    ok = ok && fabsf(b) <= 65504.0f && fabsf(fmaf(15.0f, s, b)) <= 65504.0f;
  }
  return ok;
}

// Dequantize NC 16-byte code chunks (32 elements each, starting at chunk c0 of the row) of
// one key into its row of a swizzled operand tile: 8-element chunk cc of key `key` lives in
// slab cc / 8 (SLAB bytes each), row key (128 bytes), 16-byte unit (cc % 8) ^ (key % 8) --
// the layout a 128-byte-swizzled TMA load of fp16 rows produces.  F16: f16x2 arithmetic
// (every group of the row inside fp16's range); otherwise the fp32 path that saturates.
template <int NC, int SLAB, bool F16>
__device__ __forceinline__ void q4_store_key(uint8_t* tile, const uint4 (&codes)[NC],
                                             const uint32_t (&sb)[NC / 2], int key, int c0,
                                             bool sbf16) {
#pragma unroll
  for (int g = 0; g < NC / 2; ++g) {
    float s, b;
    uint32_t s2 = 0, b2 = 0;
    if constexpr (F16) {
      if (sbf16) {
        q4_group_f32(sb[g], true, s, b);
        s2 = pack_half2(s, s);
        b2 = pack_half2(b, b);
      } else {
        s2 = __byte_perm(sb[g], 0u, 0x1010);
        b2 = __byte_perm(sb[g], 0u, 0x3232);
      }
    } else {
      q4_group_f32(sb[g], sbf16, s, b);
    }
#pragma unroll
    for (int c = 2 * g; c < 2 * g + 2; ++c) {
      const uint32_t w[4] = {codes[c].x, codes[c].y, codes[c].z, codes[c].w};
#pragma unroll
      for (int wi = 0; wi < 4; ++wi) {
        const int cc = (c0 + c) * 4 + wi;
        const int off = (cc / 8) * SLAB + key * 128 + (((cc % 8) ^ (key & 7)) << 4);
        *reinterpret_cast<uint4*>(tile + off) = F16 ? q4_word_f16(w[wi], s2, b2) : q4_word_f32(w[wi], s, b);
      }
    }
  }
}

// One key's share of a V tile as the dequantizing threads hold it: NC 16-byte code chunks and
// the (scale | bias << 16) words of their NC / 2 groups.
template <int NC>
struct Q4Row {
  uint4 v[NC];
  uint32_t sb[NC / 2];
};

// The saturating fp32 conversion of a row, out of line: it runs only for rows with a group
// beyond fp16's range, and keeping its code out of the streaming loop leaves the
// instruction cache to the common path.
template <int NC, int SLAB>
__device__ __noinline__ void q4_store_key_saturating(uint8_t* tile, Q4Row<NC> r, int key, int c0,
                                                     bool sbf16) {
  q4_store_key<NC, SLAB, false>(tile, r.v, r.sb, key, c0, sbf16);
}

// Element of its 8-element chunk that column `col` of O holds (position 2i: element i,
// position 2i + 1: element i + 4).
__host__ __device__ constexpr int q4_chunk_elem(int col) {
  return (col & ~7) | ((col & 1) << 2) | ((col >> 1) & 3);
}

// ---------------------------------------------------------------- attention kernel
// Softmax geometry: CG = BN / CPW warps share each TMEM lane quarter (32 query rows), each
// owning CPW key columns of every tile, so 4 CG softmax warps overlap one another's
// TMEM-load, exponential and barrier latencies.
// Warp 4 CG streams K/V tiles (TMA) and warp 4 CG + 1 issues the MMAs.
// Key columns each softmax warp owns per tile (32 or 64): fewer columns mean more warps per
// SM sub-partition to overlap latencies, more columns less fixed cost per score.
constexpr int kPrefillColsPerWarp = 64;

template <int BN>
struct SoftmaxGeom {
  static constexpr int CPW = BN / 2 < kPrefillColsPerWarp ? BN / 2 : kPrefillColsPerWarp;
  static constexpr int CG = BN / CPW;
  static constexpr int WARPS = 4 * CG;
  static constexpr int THREADS = 32 * WARPS;
  static constexpr int TMA_WARP = WARPS, MMA_WARP = WARPS + 1;
  static constexpr int CTA_THREADS = THREADS + 64;
};

// Warp roles of the one-tile kernel: softmax warps, the TMA thread's warp, kVDequantWarps
// warps that dequantize V tiles from the Q4 cache (QV4), then the MMA thread's warp.
constexpr int kVDequantWarps = 4;

// Head dims whose V tiles are dequantized in the attention kernel (the stage kernel then
// writes only the K plane): MLA's 192 / 128, where it measured ~2% faster per layer and
// saves the V plane (0.57 GB at B 16, 16 heads, 8704 keys).  Gemma-3's 256 / 256 (64-key
// tiles, two threads per key) measured 2-4% slower and keeps the stage for V.
template <int DK, int DV>
constexpr bool kPrefillVInKernel = DK == 192 && DV == 128;

template <int BN, bool QV4>
struct PrefillRoles {
  static constexpr int TMA_WARP = SoftmaxGeom<BN>::WARPS;
  static constexpr int DQ_WARP = TMA_WARP + 1;
  static constexpr int MMA_WARP = DQ_WARP + (QV4 ? kVDequantWarps : 0);
  static constexpr int THREADS = 32 * (MMA_WARP + 1);
};

template <int DK, int DV, int BN, int NS, int NSV>
struct PrefillLayout {
  static constexpr int CG = SoftmaxGeom<BN>::CG;
  static constexpr int QSLAB = 128 * 128;  // 128 query rows x 64 fp16 (one swizzled slab)
  static constexpr int KSLAB = BN * 128;   // BN keys x 64 fp16
  static constexpr int VSLAB = BN * 128;
  static constexpr int KSTAGE = (DK / 64) * KSLAB;
  static constexpr int VSTAGE = (DV / 64) * VSLAB;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + (DK / 64) * QSLAB;
  static constexpr int OFF_V = OFF_K + NS * KSTAGE;
  static constexpr int OFF_QF = OFF_V + NSV * VSTAGE;  // per-row query factor (128 floats)
  static constexpr int OFF_RX = OFF_QF + 128 * 4;     // row exchange between column groups [CG][128]
  static constexpr int OFF_BAR = OFF_RX + CG * 128 * 4;
  // mbarriers: K full / empty (NS each), V full / empty (NSV each), S full x2, P full x2,
  // O full x2, drain.  Every barrier that completes once per tile alternates between two
  // copies by tile parity, so a parity wait can never be satisfied by the phase of the tile
  // before last.
  static constexpr int B_KFULL = 0, B_KEMPTY = NS, B_VFULL = 2 * NS, B_VEMPTY = 2 * NS + NSV;
  static constexpr int B_SFULL = 2 * NS + 2 * NSV, B_PFULL = B_SFULL + 2;
  static constexpr int B_OFULL = B_PFULL + 2, B_DRAIN = B_OFULL + 2, B_COUNT = B_DRAIN + 1;
  static constexpr int SMEM = OFF_BAR + B_COUNT * 8 + 16;  // + TMEM slot and abort flag
  static constexpr uint32_t TMEM_COLS = 512;  // S x2 (2 BN) + O (DV)
  static constexpr int O_COL = 2 * BN;
  static_assert(DK % 64 == 0 && DV % 64 == 0 && DK <= 256 && DV <= 256, "head dims");
  static_assert(BN == 64 || BN == 128, "key tiles of 64 or 128");
  static_assert(2 * BN + DV <= 512, "S x2 + O must fit in TMEM");
  static_assert((DV / CG) % 16 == 0, "O columns per softmax warp");
};

// Named barrier over `count` threads that also ORs a flag across them: every thread gets the
// same answer, so the warps of a lane quarter leave their loop together even if the shared
// abort flag changes while their threads read it.
__device__ __forceinline__ bool group_bar_any(int id, bool v, int count) {
  uint32_t r;
  asm volatile(
      "{\n.reg .pred p, q;\nsetp.ne.u32 p, %1, 0;\nbar.red.or.pred q, %2, %3, p;\n"
      "selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

// Bounded wait that also gives up as soon as another role of the CTA raised the abort flag.
__device__ __forceinline__ bool wait_or_abort(uint32_t bar, uint32_t parity, uint64_t limit_ns,
                                              const volatile int* abort_flag) {
  if (limit_ns == 0) return false;
  constexpr uint32_t kSuspendNs = 100000;
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
    if (*abort_flag) return false;
    if (it == 0) {
      t0 = globaltimer_ns();
    } else if (globaltimer_ns() - t0 > limit_ns) {
      return false;
    }
  }
}

// Multiply this thread's TMEM row of O (NC columns at taddr) by f.
template <int NC>
__device__ __forceinline__ void rescale_o(uint32_t taddr, float f) {
  constexpr int C = NC < 32 ? NC : 32;
#pragma unroll 1
  for (int c = 0; c < NC / C; ++c) {
    float v[C];
    tc::tmem_ld<C>(taddr + c * C, v);
#pragma unroll
    for (int j = 0; j < C; ++j) v[j] *= f;
    tc::tmem_stf<C>(taddr + c * C, v);
  }
}

template <int DK, int DV, int BN, int NS, int NSV, bool DENSE, bool QV4>
__global__ void __launch_bounds__(PrefillRoles<BN, QV4>::THREADS, 1)
    prefill_kernel(const __grid_constant__ DecodeParams p) {
  using LY = PrefillLayout<DK, DV, BN, NS, NSV>;
  using SG = SoftmaxGeom<BN>;
  using RL = PrefillRoles<BN, QV4>;
  static_assert(LY::SMEM <= 232448, "dynamic shared memory of one CTA");
  constexpr int CG = SG::CG;
  constexpr int CPW = SG::CPW;
  constexpr int KSTEPS = DK / 16;  // S = Q . K^T: 16-deep steps over the head dim
  constexpr int PSTEPS = BN / 16;  // O += P . V: 16 keys per step
  constexpr int DH = DV / CG;      // O columns each softmax warp rescales and stores

  // The swizzled operand tiles need a 1024-byte aligned window: refuse (every thread alike,
  // before any barrier or TMEM allocation) rather than feed the tensor cores a shifted pattern.
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t s_base = smem_u32(smem);
  if (s_base & 1023u) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
      flag_status(p.status, AM_STATUS_BAD_POSITION);
    return;
  }
  const uint32_t sQ = s_base + LY::OFF_Q, sK = s_base + LY::OFF_K, sV = s_base + LY::OFF_V;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LY::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + LY::OFF_BAR + LY::B_COUNT * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + LY::OFF_BAR + LY::B_COUNT * 8 + 4);
  float* sqf = reinterpret_cast<float*>(smem + LY::OFF_QF);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  // Grid (query tile, KV head, sequence) with the query tile fastest: the CTAs that stream
  // the same K/V plane run side by side, so each tile of the plane comes from DRAM once and
  // from L2 for the others (with the query tile slowest, a plane larger than a share of L2
  // was read from DRAM once per query tile).  Reversed, so the causal tiles that see the
  // most keys start first.
  const int h = blockIdx.y, b = blockIdx.z;
  const int n_rep = p.n_rep;
  const int tok_per_cta = 128 / n_rep;
  const int l0 = (gridDim.x - 1 - blockIdx.x) * tok_per_cta;
  const int l_last = min(l0 + tok_per_cta, p.q_len) - 1;

  const int n = p.kv_len[b];
  const int st = p.kv_start != nullptr ? p.kv_start[b] : 0;
  int blo, bhi;  // the workspace plane holds keys [blo, blo + nw)
  prefill_block_range(p, b, blo, bhi);
  bhi = min(bhi, blo + p.nw);
  const int pos_min = n - p.q_len + l0, pos_max = n - p.q_len + l_last;
  int lo = blo, hi = bhi;  // keys this CTA's rows can see
  if (!DENSE && p.window > 0) lo = max(lo, pos_min - p.window + 1);
  if (p.causal) hi = min(hi, pos_max + 1);
  const int n_tiles = hi > lo ? (hi - lo + BN - 1) / BN : 0;

  // ---- setup
  if (tid == 0) {
    for (int i = 0; i < LY::B_COUNT; ++i) {
      const bool pfull = i == LY::B_PFULL || i == LY::B_PFULL + 1;
      const bool vfull = i >= LY::B_VFULL && i < LY::B_VFULL + NSV;  // QV4: one arrival per dequantizing thread
      mbar_init(bar(i), pfull ? SG::THREADS : (QV4 && vfull) ? 32 * kVDequantWarps : 1);
    }
    fence_mbar_init();
    *abort_flag = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(LY::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  if (tid < 256) {
    // query row r -> fp16 with a power-of-two prescale (exact for fp16 / bf16 inputs); two
    // threads per row (adjacent lanes), each staging half of it
    const int r = tid >> 1, half = tid & 1;
    constexpr int CH = DK / 16;
    const int rl = r / n_rep;
    const bool row_ok = r < tok_per_cta * n_rep && l0 + rl < p.q_len;
    const int l = l0 + (row_ok ? rl : 0);
    const int hq = h * n_rep + r % n_rep;
    const uint16_t* qrow = p.q + (int64_t)b * p.qsb + (int64_t)hq * p.qsh + (int64_t)l * p.qsl;
    uint4 raw[CH];
    q_chunks_load<CH>(qrow + half * (DK / 2), row_ok, raw);
    float amax = q_chunks_amax<CH>(raw, p.q_bf16 != 0);
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    const float pw = q_row_prescale(amax, p.scale_log2);
    if (half == 0) sqf[r] = p.scale_log2 / pw;
    q_chunks_store<CH>(smem + LY::OFF_Q, LY::QSLAB, raw, pw, p.q_bf16 != 0, r, half * CH);
  }
  fence_proxy_async_smem();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr uint32_t ID_S = tc::idesc(128, BN, false);
  constexpr uint32_t ID_O = tc::idesc(128, DV, true);

  int issued_k = 0, issued_v = 0;  // TMA thread: tiles whose loads were issued
  bool mma_issued = false;         // MMA thread: any tcgen05.mma issued

  if (warp == RL::TMA_WARP) {
    // ================================================================ TMA producer
    if (lane == 0 && n_tiles > 0) {
      griddep_wait();  // the stage kernel's workspace rows are complete and visible
      const int y0 = (b * p.hkv + h) * p.nw + (lo - blo);
      bool ok = true;
      for (int j = 0; j < n_tiles; ++j) {
        const int s = j % NS;
        if (j >= NS) ok = wait_or_abort(bar(LY::B_KEMPTY + s), ((j - NS) / NS) & 1, p.wait_ns, abort_flag);
        if (!ok) break;
        mbar_arrive_expect_tx(bar(LY::B_KFULL + s), LY::KSTAGE);
#pragma unroll
        for (int x = 0; x < DK / 64; ++x)
          tma_load_2d(sK + s * LY::KSTAGE + x * LY::KSLAB, &p.tmap_kd, x * 128, y0 + j * BN,
                      bar(LY::B_KFULL + s));
        issued_k = j + 1;
        if constexpr (QV4) continue;  // V tiles come from the dequantizing warps
        const int sv = j % NSV;
        if (j >= NSV) ok = wait_or_abort(bar(LY::B_VEMPTY + sv), ((j - NSV) / NSV) & 1, p.wait_ns, abort_flag);
        if (!ok) break;
        mbar_arrive_expect_tx(bar(LY::B_VFULL + sv), LY::VSTAGE);
#pragma unroll
        for (int x = 0; x < DV / 64; ++x)
          tma_load_2d(sV + sv * LY::VSTAGE + x * LY::VSLAB, &p.tmap_vd, x * 128, y0 + j * BN,
                      bar(LY::B_VFULL + sv));
        issued_v = j + 1;
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (QV4 && warp >= RL::DQ_WARP && warp < RL::MMA_WARP) {
    // ================================================================ V dequantizing producer
    // 128 threads, one (BN = 128) or two (BN = 64) per key of a tile: each keeps the code
    // chunks, scales and biases of its key for three tiles in registers, loading tile j + 2
    // before it converts tile j into the V ring, then arrives on the slot's full barrier.
    if constexpr (QV4) {
      static_assert(32 * kVDequantWarps == 128 && 128 % BN == 0, "one or two threads per key");
      constexpr int TPK = 128 / BN;
      constexpr int VC = DV / 32 / TPK;  // 16-byte code chunks (32 elements) per thread
      static_assert(VC % 2 == 0, "whole 64-element groups per thread");
      constexpr int NGV = DV / 64;
      const int dt = tid - 32 * RL::DQ_WARP;
      const int kk = dt % BN, part = dt / BN;
      const bool sbf16 = p.scale_bf16 != 0;
      using Raw = Q4Row<VC>;
      auto load = [&](int j, Raw& r) {
        const int t = lo + j * BN + kk;
        int64_t row = -1;
        if (t < hi) {
          if (p.paged) {
            const int blk_i = t / p.block_tokens;
            const int32_t blk = blk_i < p.table_stride ? p.table[(int64_t)b * p.table_stride + blk_i] : -1;
            if (blk < 0 || blk >= p.capacity) {
              flag_status(p.status, AM_STATUS_BAD_BLOCK);
            } else {
              row = ((int64_t)blk * p.hkv + h) * p.block_tokens + t % p.block_tokens;
            }
          } else if (t < p.capacity) {
            row = ((int64_t)b * p.hkv + h) * p.capacity + t;
          } else {
            flag_status(p.status, AM_STATUS_BAD_POSITION);
          }
        }
        if (row >= 0) {
          const uint4* vc = reinterpret_cast<const uint4*>(p.vc + row * (DV / 8)) + part * VC;
#pragma unroll
          for (int c = 0; c < VC; ++c) r.v[c] = __ldg(vc + c);
#pragma unroll
          for (int g2 = 0; g2 < VC / 2; ++g2) {
            const int64_t gi = row * NGV + part * (VC / 2) + g2;
            r.sb[g2] = static_cast<uint32_t>(__ldg(p.vs + gi)) | (static_cast<uint32_t>(__ldg(p.vb + gi)) << 16);
          }
        } else {  // past the visible keys or behind a bad block: a zero row (scale = bias = 0)
#pragma unroll
          for (int c = 0; c < VC; ++c) r.v[c] = make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int g2 = 0; g2 < VC / 2; ++g2) r.sb[g2] = 0;
        }
      };
      auto put = [&](int j, const Raw& r) -> bool {
        const int sv = j % NSV;
        // the range test runs before the ring-slot wait, off the slot-free -> P . V chain
        const bool in_range = q4_groups_in_f16_range(r.sb, sbf16);
        if (j >= NSV &&
            !wait_or_abort(bar(LY::B_VEMPTY + sv), ((j - NSV) / NSV) & 1, p.wait_ns, abort_flag))
          return false;
        uint8_t* tile = smem + LY::OFF_V + sv * LY::VSTAGE;
        // (the lanes still here vote: a lane that gave up on the wait has left)
        if (__all_sync(__activemask(), in_range)) {
          q4_store_key<VC, LY::VSLAB, true>(tile, r.v, r.sb, kk, part * VC, sbf16);
        } else {  // a group leaves fp16's range: saturate it as the stage kernel does
          q4_store_key_saturating<VC, LY::VSLAB>(tile, r, kk, part * VC, sbf16);
        }
        fence_proxy_async_smem();  // the tensor core reads the tile through the async proxy
        mbar_arrive(bar(LY::B_VFULL + sv));
        return true;
      };
      if (n_tiles > 0) {
        griddep_wait();  // the cache rows are complete and visible
        Raw r0, r1, r2;
        load(0, r0);
        if (1 < n_tiles) load(1, r1);
        bool ok = true;
        for (int j = 0; j < n_tiles; j += 3) {
          if (j + 2 < n_tiles) load(j + 2, r2);
          ok = put(j, r0);
          if (!ok || j + 1 >= n_tiles) break;
          if (j + 3 < n_tiles) load(j + 3, r0);
          ok = put(j + 1, r1);
          if (!ok || j + 2 >= n_tiles) break;
          if (j + 4 < n_tiles) load(j + 4, r1);
          ok = put(j + 2, r2);
          if (!ok) break;
        }
        if (!ok) *abort_flag = 1;
      }
    }
  } else if (warp == RL::MMA_WARP) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      bool ok = true;
      for (int j = 0; j <= n_tiles; ++j) {
        if (j < n_tiles) {
          const int s = j % NS, buf = j & 1;
          ok = wait_or_abort(bar(LY::B_KFULL + s), (j / NS) & 1, p.wait_ns, abort_flag);
          // S[buf] holds P of tile j - 2: the P . V that reads it was issued before (in the
          // previous iteration), and tcgen05.mma operations from one thread execute in issue
          // order, so S_j is issued without waiting for that P . V to complete
          if (!ok) break;
          tc::fence_after();
          const uint32_t kst = sK + s * LY::KSTAGE;
#pragma unroll
          for (int ks = 0; ks < KSTEPS; ++ks) {
            tc::mma(tmem + buf * BN,
                    tc::sdesc(sQ + (ks / 4) * LY::QSLAB + (ks % 4) * 32, 16, 1024),
                    tc::sdesc(kst + (ks / 4) * LY::KSLAB + (ks % 4) * 32, 16, 1024), ID_S,
                    ks > 0 ? 1u : 0u);
          }
          mma_issued = true;
          tc::commit(bar(LY::B_SFULL + buf));
          tc::commit(bar(LY::B_KEMPTY + s));
        }
        if (j >= 1) {
          const int jj = j - 1, s = jj % NSV, buf = jj & 1;
          ok = wait_or_abort(bar(LY::B_VFULL + s), (jj / NSV) & 1, p.wait_ns, abort_flag);
          if (ok) ok = wait_or_abort(bar(LY::B_PFULL + buf), (jj >> 1) & 1, p.wait_ns, abort_flag);
          if (!ok) break;
          tc::fence_after();
          const uint32_t vst = sV + s * LY::VSTAGE;
#pragma unroll
          for (int ks = 0; ks < PSTEPS; ++ks) {
            // keys 16 ks .. +15: P pairs of column group ks / (CPW / 16) (CPW keys in CPW / 2
            // P columns each)
            const int pcol = (ks / (CPW / 16)) * CPW + (ks % (CPW / 16)) * 8;
            tc::mma_ts(tmem + LY::O_COL, tmem + buf * BN + pcol,
                       tc::sdesc(vst + ks * 2048, LY::VSLAB, 1024), ID_O, (jj > 0 || ks > 0) ? 1u : 0u);
          }
          tc::commit(bar(LY::B_OFULL + buf));
          tc::commit(bar(LY::B_VEMPTY + s));
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ================================================================ softmax warps
    // Warp w owns S rows 32 (w % 4) .. +31 (its TMEM lane quarter) and key columns
    // CPW (w / 4) .. +CPW-1 of every tile; the CG warps of a quarter exchange their row maxima
    // through shared memory (a named barrier per quarter) and keep partial sums that are
    // added at the end.  Each also rescales and writes back DV / CG columns of O.
    const int quarter = warp & 3, cg = warp >> 2;
    const int r = quarter * 32 + lane;     // query row == TMEM lane
    const int qbar = 1 + quarter;          // named barrier of the quarter's CG warps
    constexpr int QBAR_THREADS = 32 * CG;
    const int rl = r / n_rep;
    const bool row_ok = r < tok_per_cta * n_rep && l0 + rl < p.q_len;
    const int l = l0 + (row_ok ? rl : 0);
    const int hq = h * n_rep + r % n_rep;
    const int pos = n - p.q_len + l;
    // (keys past the workspace plane, bhi, exist only when kv_len exceeds the max_kv_len the
    // call was sized for: they are masked, and the status word says so)
    const int klo = max(st, p.window > 0 ? pos - p.window + 1 : 0);
    const int khi = min(p.causal ? min(n, pos + 1) : n, bhi);
    // keys every row of the CTA sees (tiles inside need no per-element mask)
    const int tlo = max(st, p.window > 0 ? pos_max - p.window + 1 : 0);
    const int thi = min(p.causal ? min(n, pos_min + 1) : n, bhi);
    const float q_fac = sqf[r];
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    float* rx = reinterpret_cast<float*>(smem + LY::OFF_RX);  // [CG][128]

    float m_run = -INFINITY, l_run = 0.0f;
    const uint32_t o_row = tmem + LY::O_COL + lane_base;  // this thread's row of O
    auto masked = [&](float s, int tok) -> float {
      if (!(row_ok && tok >= klo && tok < khi)) return -INFINITY;
      if constexpr (DENSE) {
        const int64_t idx = (int64_t)b * p.msb + (int64_t)hq * p.msh + (int64_t)l * p.msl +
                            (int64_t)tok * p.msn;
        if (p.mask_kind == AM_MASK_BOOL) {
          if (static_cast<const uint8_t*>(p.mask)[idx] == 0) return -1.0e30f;
        } else {
          const float mv = p.mask_dtype == AM_DTYPE_F32
                               ? static_cast<const float*>(p.mask)[idx]
                               : h2f_rt(static_cast<const uint16_t*>(p.mask)[idx],
                                        p.mask_dtype == AM_DTYPE_BF16);
          s = fmaf(mv, 1.4426950408889634f, s);
        }
      }
      return s;
    };

    for (int i = 0; i < n_tiles; ++i) {
      const int buf = i & 1;
      const int t0 = lo + i * BN + cg * CPW;  // first key of this warp's columns
      bool ok = !*abort_flag && wait_or_abort(bar(LY::B_SFULL + buf), (i >> 1) & 1, p.wait_ns, abort_flag);
      // (this barrier also keeps every warp of the quarter from overwriting rx before the
      // others have read the previous tile's maxima)
      if (group_bar_any(qbar, !ok, QBAR_THREADS)) {
        *abort_flag = 1;
        break;
      }
      tc::fence_after();
      const bool need_mask =
          __any_sync(0xffffffffu, DENSE || !row_ok || t0 < tlo || t0 + CPW > thi);  // warp-uniform
      float v[CPW];
      tc::tmem_ld<CPW>(tmem + buf * BN + cg * CPW + lane_base, v);
      if (need_mask) {
#pragma unroll
        for (int j2 = 0; j2 < CPW; ++j2) v[j2] = masked(v[j2] * q_fac, t0 + j2);
      }
      // q_fac > 0 (the sign of the softmax scale lives in the query tile), so the row max of
      // the raw scores is the max of the scaled ones
      float mp[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mp[k] = v[k];
#pragma unroll
      for (int j2 = 8; j2 < CPW; ++j2) mp[j2 & 7] = fmaxf(mp[j2 & 7], v[j2]);
#pragma unroll
      for (int k = 1; k < 8; ++k) mp[0] = fmaxf(mp[0], mp[k]);
      const float my_max = need_mask ? mp[0] : mp[0] * q_fac;
      rx[cg * 128 + r] = my_max;
      if (group_bar_any(qbar, false, QBAR_THREADS)) {  // publishes rx within the quarter
        *abort_flag = 1;
        break;
      }
      float tile_max = rx[r];
#pragma unroll
      for (int g2 = 1; g2 < CG; ++g2) tile_max = fmaxf(tile_max, rx[g2 * 128 + r]);
      const bool raise = tile_max > m_run + kPrefillRescaleSlack;
      if (__any_sync(0xffffffffu, raise)) {  // the same rows, so the same answer in every group
        const float m_new = raise ? tile_max : m_run;
        const float alpha = m_run == -INFINITY ? 0.0f : ex2(m_run - m_new);
        if (i >= 1) {
          // O is rescaled in TMEM only after P . V of the previous tile has landed in it
          const int pv = i - 1;
          if (__all_sync(0xffffffffu, wait_or_abort(bar(LY::B_OFULL + (pv & 1)), (pv >> 1) & 1,
                                                    p.wait_ns, abort_flag))) {
            tc::fence_after();
            rescale_o<DH>(o_row + cg * DH, alpha);
          } else {
            *abort_flag = 1;
          }
        }
        l_run *= alpha;
        m_run = m_new;
      }
      const float m_safe = m_run == -INFINITY ? 0.0f : m_run;
      const float fac = need_mask ? 1.0f : q_fac;  // masked scores already carry q_fac
      float lp[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) lp[k] = 0.0f;
      // P (fp16 pairs) replaces this warp's own S columns: keys cg * CPW + 2c, +1 in column
      // cg * CPW + c of the tile's S buffer, the A operand of P . V
      uint32_t pk[CPW / 2];
#pragma unroll
      for (int c = 0; c < CPW / 2; ++c) {
        const float x0 = fmaf(v[2 * c], fac, -m_safe);
        const float x1 = fmaf(v[2 * c + 1], fac, -m_safe);
        float p0 = 0.0f, p1 = 0.0f;
        bool fma_exp = false;
        if constexpr (kFmaExpEvery > 0) fma_exp = (c % (kFmaExpEvery > 0 ? kFmaExpEvery : 1)) == kFmaExpEvery - 1;
        if (fma_exp) {
          p0 = ex2_fma(x0);
          p1 = ex2_fma(x1);
        } else {
          p0 = ex2(x0);
          p1 = ex2(x1);
        }
        lp[(2 * c) & 7] += p0;
        lp[(2 * c + 1) & 7] += p1;
        pk[c] = pack_half2(p0, p1);
      }
      tc::tmem_st<CPW / 2>(tmem + buf * BN + cg * CPW + lane_base, pk);
#pragma unroll
      for (int k = 0; k < 8; ++k) l_run += lp[k];
      tc::fence_before();
      mbar_arrive(bar(LY::B_PFULL + buf));
    }
    // ---- epilogue: this thread's DV / CG columns of its output row.  P . V of the last tile
    // (and, by the order of commits, of every earlier tile) must have landed in O.  The
    // quarter adds its partial sums; the first OR barrier makes sure every warp has read the
    // last tile's maxima from rx before the partial sums overwrite them.
    bool fin = !*abort_flag;
    if (fin && n_tiles > 0) {
      const int pv = n_tiles - 1;
      fin = wait_or_abort(bar(LY::B_OFULL + (pv & 1)), (pv >> 1) & 1, p.wait_ns, abort_flag);
    }
    fin = __all_sync(0xffffffffu, fin);
    const bool bad0 = group_bar_any(qbar, !fin, QBAR_THREADS);
    rx[cg * 128 + r] = l_run;
    const bool bad = group_bar_any(qbar, bad0, QBAR_THREADS);
    if (!bad) {
      tc::fence_after();
      // 32 columns at a time (DH is up to 128 fp32 accumulators per thread)
      float inv = 0.0f;
      if (row_ok) {
        float l_tot = 0.0f;
#pragma unroll
        for (int g2 = 0; g2 < CG; ++g2) l_tot += rx[g2 * 128 + r];
        const bool sink = p.sinks != nullptr;
        inv = softmax_out_factor(m_run, l_tot, sink, sink ? p.sinks[hq] * 1.4426950408889634f : 0.0f);
      }
      const int64_t ob = (int64_t)b * p.osb + (int64_t)hq * p.osh + (int64_t)l * p.osl + cg * DH;
      constexpr int C = DH < 32 ? DH : 32;
#pragma unroll 1
      for (int c = 0; c < DH / C; ++c) {
        float o_acc[C];
        if (n_tiles > 0) {
          float tcv[C];
          __syncwarp();  // tcgen05.ld is warp-collective: converge after the previous chunk's stores
          tc::tmem_ld<C>(o_row + cg * DH + c * C, tcv);
#pragma unroll
          for (int j2 = 0; j2 < C; ++j2)  // (QV4: columns back in element order)
            o_acc[QV4 ? q4_chunk_elem(j2) : j2] = tcv[j2];
        } else {
#pragma unroll
          for (int j2 = 0; j2 < C; ++j2) o_acc[j2] = 0.0f;
        }
        if (!row_ok) continue;  // (no collective below)
        if (p.out_dtype == AM_DTYPE_F32) {
          float* o = static_cast<float*>(p.out) + ob + c * C;
          if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
            for (int d = 0; d < C; d += 4)
              *reinterpret_cast<float4*>(o + d) =
                  make_float4(o_acc[d] * inv, o_acc[d + 1] * inv, o_acc[d + 2] * inv, o_acc[d + 3] * inv);
          } else {
#pragma unroll
            for (int d = 0; d < C; ++d) o[d] = o_acc[d] * inv;
          }
        } else {
          const bool bf = p.out_dtype == AM_DTYPE_BF16;
          uint16_t* o = static_cast<uint16_t*>(p.out) + ob + c * C;
          if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
            for (int d = 0; d < C; d += 8) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float a = o_acc[d + 2 * e] * inv, c2 = o_acc[d + 2 * e + 1] * inv;
                w[e] = bf ? (static_cast<uint32_t>(f2h<true>(a)) | (static_cast<uint32_t>(f2h<true>(c2)) << 16))
                          : pack_half2(a, c2);
              }
              *reinterpret_cast<uint4*>(o + d) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          } else {
#pragma unroll
            for (int d = 0; d < C; ++d) o[d] = bf ? f2h<true>(o_acc[d] * inv) : f2h<false>(o_acc[d] * inv);
          }
        }
      }
    } else {
      *abort_flag = 1;
    }
  }

  // ---- teardown: after an abort, let this CTA's TMA loads and MMAs in flight finish
  // (bounded) before the shared memory and TMEM are released.
  __syncthreads();
  if (*abort_flag) {
    constexpr uint64_t kDrainNs = 100000000ull;
    if (warp == RL::TMA_WARP && lane == 0) {
      for (int jj = max(0, issued_k - NS); jj < issued_k; ++jj)
        mbar_wait_bounded(bar(LY::B_KFULL + jj % NS), (jj / NS) & 1, kDrainNs);
      for (int jj = max(0, issued_v - NSV); jj < issued_v; ++jj)  // (QV4: none issued)
        mbar_wait_bounded(bar(LY::B_VFULL + jj % NSV), (jj / NSV) & 1, kDrainNs);
    }
    if (warp == RL::MMA_WARP && lane == 0 && mma_issued) {
      tc::commit(bar(LY::B_DRAIN));
      mbar_wait_bounded(bar(LY::B_DRAIN), 0, kDrainNs);
    }
    if (tid == 0) flag_status(p.status, AM_STATUS_TIMEOUT);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                 "r"(LY::TMEM_COLS));
  }
}

// 64 scores of one row -> 32 fp16 P pairs stored to TMEM at taddr (keys 2c, 2c + 1 in
// column c), the exponentials added into ls: x = s * fac - m on packed fp32 pairs, a fixed
// share of the 2^x through the FMA-pipe polynomial.
// The same without the store: the 32 packed pairs are returned in pk.
__device__ __forceinline__ void softmax_pack(const float (&v)[64], float2 fac2, float2 nm2,
                                             float2 (&ls)[4], uint32_t (&pk)[32]) {
#pragma unroll
  for (int c = 0; c < 32; ++c) {
    const float2 x = __ffma2_rn(make_float2(v[2 * c], v[2 * c + 1]), fac2, nm2);
    bool fma_exp = false;
    if constexpr (kTile2FmaExpEvery > 0)
      fma_exp = (c % (kTile2FmaExpEvery > 0 ? kTile2FmaExpEvery : 1)) == kTile2FmaExpEvery - 1;
    const float2 pr = fma_exp ? ex2_fma2(x) : make_float2(ex2(x.x), ex2(x.y));
    ls[c & 3] = __fadd2_rn(ls[c & 3], pr);
    pk[c] = pack_half2(pr.x, pr.y);
  }
}

__device__ __forceinline__ void softmax_half(const float (&v)[64], float2 fac2, float2 nm2,
                                             float2 (&ls)[4], uint32_t taddr) {
  // stored 16 columns at a time, so at most 16 packed pairs are live beside the scores
#pragma unroll
  for (int h16 = 0; h16 < 2; ++h16) {
    uint32_t pk[16];
#pragma unroll
    for (int c16 = 0; c16 < 16; ++c16) {
      const int c = 16 * h16 + c16;
      const float2 x = __ffma2_rn(make_float2(v[2 * c], v[2 * c + 1]), fac2, nm2);
      bool fma_exp = false;
      if constexpr (kTile2FmaExpEvery > 0)
        fma_exp = (c % (kTile2FmaExpEvery > 0 ? kTile2FmaExpEvery : 1)) == kTile2FmaExpEvery - 1;
      const float2 pr = fma_exp ? ex2_fma2(x) : make_float2(ex2(x.x), ex2(x.y));
      ls[c & 3] = __fadd2_rn(ls[c & 3], pr);
      pk[c16] = pack_half2(pr.x, pr.y);
    }
    tc::tmem_st16(taddr + 16 * h16, pk);
  }
}

// ---------------------------------------------------------------- two-tile attention kernel
// Head dims up to 128: one CTA holds two 128-row query tiles (qt = 0, 1: 256 query rows, 256 /
// n_rep tokens) of one KV head of one sequence, so every 128-key K/V tile fed from L2 serves
// twice the rows, and the tensor core works on one query tile while the softmax warps of the
// other run.  TMEM: S[qt] (128 columns each, P written back over it) and O[qt] (Dv columns
// each).  Softmax warps: 4 per query tile, warp w owning TMEM lane quarter w % 4 of tile
// w / 4: one thread per query row, all 128 key columns of a tile, so no exchange between
// warps.  320 threads: softmax warps 0-7, the TMA thread in warp 8, the MMA thread in warp 9
// (its issue order is described there).
constexpr int kTile2Threads = 320;

template <int DK, int DV, int NS>
struct Prefill2Layout {
  static constexpr int BN = 128;
  static constexpr int QSLAB = 128 * 128;          // 128 query rows x 64 fp16
  static constexpr int QTILE = (DK / 64) * QSLAB;  // one query tile
  static constexpr int KSLAB = BN * 128, VSLAB = BN * 128;
  static constexpr int KSTAGE = (DK / 64) * KSLAB, VSTAGE = (DV / 64) * VSLAB;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + 2 * QTILE;
  static constexpr int OFF_V = OFF_K + NS * KSTAGE;
  static constexpr int OFF_QF = OFF_V + NS * VSTAGE;  // per-row query factor (256 floats)
  static constexpr int OFF_BAR = OFF_QF + 256 * 4;
  // mbarriers: K full / empty, V full / empty (NS each); per query tile: S full, P full,
  // O full; drain
  static constexpr int B_KFULL = 0, B_KEMPTY = NS, B_VFULL = 2 * NS, B_VEMPTY = 3 * NS;
  static constexpr int B_SFULL = 4 * NS, B_PFULL = B_SFULL + 2;
  static constexpr int B_OFULL = B_PFULL + 2, B_DRAIN = B_OFULL + 2, B_COUNT = B_DRAIN + 1;
  static constexpr int SMEM = OFF_BAR + B_COUNT * 8 + 16;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int O_COL = 2 * BN;  // S[qt] at qt * BN, O[qt] at O_COL + qt * DV
  static_assert(DK <= 128 && DV <= 128 && DK % 64 == 0 && DV % 64 == 0, "head dims up to 128");
  static_assert(2 * BN + 2 * DV <= 512, "S x2 + O x2 must fit in TMEM");
};

template <int DK, int DV, int NS, bool DENSE>
__global__ void __launch_bounds__(kTile2Threads, 1) prefill2_kernel(const __grid_constant__ DecodeParams p) {
  using LY = Prefill2Layout<DK, DV, NS>;
  static_assert(LY::SMEM <= 232448, "dynamic shared memory of one CTA");
  constexpr int BN = LY::BN;
  constexpr int KSTEPS = DK / 16;  // S = Q . K^T: 16-deep steps over the head dim
  constexpr int PSTEPS = BN / 16;  // O += P . V: 16 keys per step
  constexpr int TMA_WARP = 8, MMA_WARP = 9;

  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t s_base = smem_u32(smem);
  if (s_base & 1023u) {  // swizzled tiles need a 1024-byte aligned window (every thread returns)
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
      flag_status(p.status, AM_STATUS_BAD_POSITION);
    return;
  }
  const uint32_t sQ = s_base + LY::OFF_Q, sK = s_base + LY::OFF_K, sV = s_base + LY::OFF_V;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LY::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + LY::OFF_BAR + LY::B_COUNT * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + LY::OFF_BAR + LY::B_COUNT * 8 + 4);
  float* sqf = reinterpret_cast<float*>(smem + LY::OFF_QF);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  // Grid (query block, KV head, sequence) with the query block fastest, so the CTAs that
  // stream the same K/V plane run side by side and share its tiles through L2; reversed, so
  // the causal blocks that see the most keys start first.
  const int h = blockIdx.y, b = blockIdx.z;
  const int n_rep = p.n_rep;
  const int tpq = 128 / n_rep;  // query tokens per query tile
  const int l0 = (gridDim.x - 1 - blockIdx.x) * 2 * tpq;
  const int l_last = min(l0 + 2 * tpq, p.q_len) - 1;

  const int n = p.kv_len[b];
  const int st = p.kv_start != nullptr ? p.kv_start[b] : 0;
  int blo, bhi;  // the workspace plane holds keys [blo, blo + nw)
  prefill_block_range(p, b, blo, bhi);
  bhi = min(bhi, blo + p.nw);
  const int pos_min = n - p.q_len + l0, pos_max = n - p.q_len + l_last;
  int lo = blo, hi = bhi;  // keys the CTA's rows can see
  if (!DENSE && p.window > 0) lo = max(lo, pos_min - p.window + 1);
  if (p.causal) hi = min(hi, pos_max + 1);
  const int n_tiles = hi > lo ? (hi - lo + BN - 1) / BN : 0;

  // ---- setup
  if (tid == 0) {
    for (int i = 0; i < LY::B_COUNT; ++i)
      mbar_init(bar(i), (i == LY::B_PFULL || i == LY::B_PFULL + 1) ? 128 : 1);
    fence_mbar_init();
    *abort_flag = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(LY::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  if (tid < 256) {
    // query row R = tid of the CTA (tile R / 128, row R % 128) -> fp16 with a power-of-two
    // prescale (exact for fp16 / bf16 inputs)
    const int qt = tid >> 7, r = tid & 127;
    constexpr int CH = DK / 8;
    const int rl = r / n_rep;
    const bool row_ok = r < tpq * n_rep && l0 + qt * tpq + rl < p.q_len;
    const int l = l0 + qt * tpq + (row_ok ? rl : 0);
    const int hq = h * n_rep + r % n_rep;
    const uint16_t* qrow = p.q + (int64_t)b * p.qsb + (int64_t)hq * p.qsh + (int64_t)l * p.qsl;
    uint4 raw[CH];
    q_chunks_load<CH>(qrow, row_ok, raw);
    const float pw = q_row_prescale(q_chunks_amax<CH>(raw, p.q_bf16 != 0), p.scale_log2);
    sqf[tid] = p.scale_log2 / pw;
    q_chunks_store<CH>(smem + LY::OFF_Q + qt * LY::QTILE, LY::QSLAB, raw, pw, p.q_bf16 != 0, r, 0);
  }
  fence_proxy_async_smem();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr uint32_t ID_S = tc::idesc(128, BN, false);
  constexpr uint32_t ID_O = tc::idesc(128, DV, true);

  int issued_k = 0, issued_v = 0;  // TMA thread: tiles whose loads were issued
  bool mma_issued = false;         // MMA thread: any tcgen05.mma issued

  if (warp == TMA_WARP) {
    // ================================================================ TMA producer
    if (lane == 0 && n_tiles > 0) {
      griddep_wait();  // the stage kernel's workspace rows are complete and visible
      const int y0 = (b * p.hkv + h) * p.nw + (lo - blo);
      bool ok = true;
      for (int j = 0; j < n_tiles; ++j) {
        const int s = j % NS;
        if (j >= NS) ok = wait_or_abort(bar(LY::B_KEMPTY + s), ((j - NS) / NS) & 1, p.wait_ns, abort_flag);
        if (!ok) break;
        mbar_arrive_expect_tx(bar(LY::B_KFULL + s), LY::KSTAGE);
#pragma unroll
        for (int x = 0; x < DK / 64; ++x)
          tma_load_2d(sK + s * LY::KSTAGE + x * LY::KSLAB, &p.tmap_kd, x * 128, y0 + j * BN,
                      bar(LY::B_KFULL + s));
        issued_k = j + 1;
        if (j >= NS) ok = wait_or_abort(bar(LY::B_VEMPTY + s), ((j - NS) / NS) & 1, p.wait_ns, abort_flag);
        if (!ok) break;
        mbar_arrive_expect_tx(bar(LY::B_VFULL + s), LY::VSTAGE);
#pragma unroll
        for (int x = 0; x < DV / 64; ++x)
          tma_load_2d(sV + s * LY::VSTAGE + x * LY::VSLAB, &p.tmap_vd, x * 128, y0 + j * BN,
                      bar(LY::B_VFULL + s));
        issued_v = j + 1;
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == MMA_WARP) {
    // ================================================================ MMA issuer
    // Staggered order per key tile i: S[0]_i, O[1] += P[1]_{i-1} . V_{i-1}, S[1]_i,
    // O[0] += P[0]_i . V_i, so each query tile's softmax overlaps two MMAs of the other tile.
    // S[qt]_i overwrites the TMEM columns that held P[qt]_{i-1}: the P . V that reads them was
    // issued earlier by this thread, and tcgen05.mma operations from one thread execute in
    // issue order.  A commit arrives once every operation issued before it has completed, so
    // "S full" of tile i also means P . V of tile i - 1 has landed in O.
    if (lane == 0) {
      bool ok = true;
      auto issue_s = [&](int qt, int j) {
        const uint32_t kst = sK + (j % NS) * LY::KSTAGE;
#pragma unroll
        for (int ks = 0; ks < KSTEPS; ++ks) {
          tc::mma(tmem + qt * BN,
                  tc::sdesc(sQ + qt * LY::QTILE + (ks / 4) * LY::QSLAB + (ks % 4) * 32, 16, 1024),
                  tc::sdesc(kst + (ks / 4) * LY::KSLAB + (ks % 4) * 32, 16, 1024), ID_S,
                  ks > 0 ? 1u : 0u);
        }
        mma_issued = true;
        tc::commit(bar(LY::B_SFULL + qt));
      };
      auto issue_pv = [&](int qt, int jj) {  // after P[qt]_jj is written and V_jj has landed
        bool w = wait_or_abort(bar(LY::B_PFULL + qt), jj & 1, p.wait_ns, abort_flag);
        if (w && qt == 0) w = wait_or_abort(bar(LY::B_VFULL + jj % NS), (jj / NS) & 1, p.wait_ns, abort_flag);
        if (!w) return false;
        tc::fence_after();
        const uint32_t vst = sV + (jj % NS) * LY::VSTAGE;
#pragma unroll
        for (int ks = 0; ks < PSTEPS; ++ks) {
          // keys 16 ks .. +15: their P pairs sit in columns 8 ks .. +7 of S[qt]
          tc::mma_ts(tmem + LY::O_COL + qt * DV, tmem + qt * BN + ks * 8,
                     tc::sdesc(vst + ks * 2048, LY::VSLAB, 1024), ID_O, (jj > 0 || ks > 0) ? 1u : 0u);
        }
        tc::commit(bar(LY::B_OFULL + qt));
        return true;
      };
      for (int i = 0; i < n_tiles && ok; ++i) {
        ok = wait_or_abort(bar(LY::B_KFULL + i % NS), (i / NS) & 1, p.wait_ns, abort_flag);
        if (!ok) break;
        tc::fence_after();
        issue_s(0, i);
        if (i >= 1) {
          ok = issue_pv(1, i - 1);
          if (!ok) break;
          tc::commit(bar(LY::B_VEMPTY + (i - 1) % NS));  // both P . V of tile i - 1 issued
        }
        issue_s(1, i);
        tc::commit(bar(LY::B_KEMPTY + i % NS));
        ok = issue_pv(0, i);
      }
      if (ok && n_tiles > 0) {
        ok = issue_pv(1, n_tiles - 1);
        if (ok) tc::commit(bar(LY::B_VEMPTY + (n_tiles - 1) % NS));
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ================================================================ softmax warps
    // Warp w: query tile qt = w / 4, TMEM lane quarter w % 4, one query row per thread, all
    // 128 key columns of every tile.
    const int qt = warp >> 2, quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int rl = r / n_rep;
    const int tl0 = l0 + qt * tpq;  // first token of this query tile
    const bool row_ok = r < tpq * n_rep && tl0 + rl < p.q_len;
    const int l = tl0 + (row_ok ? rl : 0);
    const int hq = h * n_rep + r % n_rep;
    const int pos = n - p.q_len + l;
    const int klo = max(st, p.window > 0 ? pos - p.window + 1 : 0);
    const int khi = min(p.causal ? min(n, pos + 1) : n, bhi);
    // keys every row of this query tile sees (tiles inside need no per-element mask)
    const int t_last = min(tl0 + tpq, p.q_len) - 1;
    const int tlo = max(st, p.window > 0 ? n - p.q_len + t_last - p.window + 1 : 0);
    const int thi = min(p.causal ? min(n, n - p.q_len + tl0 + 1) : n, bhi);
    const float q_fac = sqf[qt * 128 + r];
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_row = tmem + qt * BN + lane_base;               // this row of S[qt]
    const uint32_t o_row = tmem + LY::O_COL + qt * DV + lane_base;   // this row of O[qt]

    float m_run = -INFINITY, l_run = 0.0f;
    auto masked = [&](float s, int tok) -> float {
      if (!(row_ok && tok >= klo && tok < khi)) return -INFINITY;
      if constexpr (DENSE) {
        const int64_t idx = (int64_t)b * p.msb + (int64_t)hq * p.msh + (int64_t)l * p.msl +
                            (int64_t)tok * p.msn;
        if (p.mask_kind == AM_MASK_BOOL) {
          if (static_cast<const uint8_t*>(p.mask)[idx] == 0) return -1.0e30f;
        } else {
          const float mv = p.mask_dtype == AM_DTYPE_F32
                               ? static_cast<const float*>(p.mask)[idx]
                               : h2f_rt(static_cast<const uint16_t*>(p.mask)[idx],
                                        p.mask_dtype == AM_DTYPE_BF16);
          s = fmaf(mv, 1.4426950408889634f, s);
        }
      }
      return s;
    };

    int done_tiles = 0;
    for (int i = 0; i < n_tiles; ++i) {
      const int t0 = lo + i * BN;
      const bool ok = !*abort_flag && wait_or_abort(bar(LY::B_SFULL + qt), i & 1, p.wait_ns, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        *abort_flag = 1;
        break;
      }
      tc::fence_after();
      const bool need_mask =
          __any_sync(0xffffffffu, DENSE || !row_ok || t0 < tlo || t0 + BN > thi);  // warp-uniform
      auto mask_half = [&](int hh, float (&v)[64]) {
        if (need_mask) {
#pragma unroll
          for (int j2 = 0; j2 < 64; ++j2) v[j2] = masked(v[j2] * q_fac, t0 + 64 * hh + j2);
        }
      };
      const float fac = need_mask ? 1.0f : q_fac;  // masked scores already carry q_fac
      const float2 fac2 = make_float2(fac, fac);
      // P against the running max as it stands, in one pass over the scores.  Every p is
      // >= 0, so a tile sum <= 2^15 bounds every p by 2^15 (inside fp16 for the P operand);
      // a larger or non-finite sum means the running max has fallen more than 15 behind, and
      // the tile is redone after a max pass (scores read once more) and a lazy rescale: the
      // running max is raised when the tile's max exceeds it by more than 2^8, so the redone
      // sum is at most 128 * 2^8.  A row with no running max yet starts with the max pass.
      // (The passes over the two 64-column halves are not unrolled: unrolled, the kernel
      // needs more registers than 320 threads get and spills.)
      bool need_max = !__all_sync(0xffffffffu, m_run != -INFINITY);
      // row max of the tile's scores (one read of S), then the lazy rescale
      auto max_pass = [&]() {
        float mp[8];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float v[64];
          tc::tmem_ld64(s_row + 64 * hh, v);
          mask_half(hh, v);
          if (hh == 0) {
#pragma unroll
            for (int k = 0; k < 8; ++k) mp[k] = v[k];
          }
#pragma unroll
          for (int j2 = hh == 0 ? 8 : 0; j2 < 64; j2 += 2)
            mp[(j2 >> 1) & 7] = max3f(mp[(j2 >> 1) & 7], v[j2], v[j2 + 1]);
        }
        mp[0] = max3f(max3f(mp[0], mp[1], mp[2]), max3f(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7]));
        const float tile_max = need_mask ? mp[0] : mp[0] * q_fac;
        const bool raise = tile_max > m_run + kPrefillRescaleSlack;
        if (__any_sync(0xffffffffu, raise)) {
          const float m_new = raise ? tile_max : m_run;
          const float alpha = m_run == -INFINITY ? 0.0f : ex2(m_run - m_new);
          if (i >= 1) {
            // P . V of the previous tile has landed in O: it read S[qt] before this tile's
            // scores were written there
            if (__all_sync(0xffffffffu, wait_or_abort(bar(LY::B_OFULL + qt), (i - 1) & 1, p.wait_ns,
                                                      abort_flag))) {
              tc::fence_after();
              rescale_o<DV>(o_row, alpha);
            } else {
              *abort_flag = 1;
            }
          }
          l_run *= alpha;
          m_run = m_new;
        }
      };
      // exponentials, row sum and P on packed fp32 pairs: x = s * fac - m, p = 2^x; P (fp16
      // pairs, keys 2c, 2c + 1 in column c: the A operand of P . V) replaces S[qt], written in
      // two halves of 32 columns
      auto exp_pass = [&]() -> float {
        const float m_safe = m_run == -INFINITY ? 0.0f : m_run;
        const float2 nm2 = make_float2(-m_safe, -m_safe);
        float2 ls[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) ls[k] = make_float2(0.0f, 0.0f);
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
          float v[64];
          tc::tmem_ld64(s_row + 64 * hh, v);
          mask_half(hh, v);
          softmax_half(v, fac2, nm2, ls, s_row + 32 * hh);
        }
        return ((ls[0].x + ls[0].y) + (ls[1].x + ls[1].y)) + ((ls[2].x + ls[2].y) + (ls[3].x + ls[3].y));
      };
      float tile_sum;
      bool done = false;
      if (!need_max) {
        // fast path: both halves' P held in registers until the sum check passes, so a
        // failed check leaves S intact for the full path
        const float2 nm2 = make_float2(-m_run, -m_run);
        float2 ls[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) ls[k] = make_float2(0.0f, 0.0f);
        uint32_t p0[32], p1[32];
        {
          float v[64];
          tc::tmem_ld64(s_row, v);
          mask_half(0, v);
          softmax_pack(v, fac2, nm2, ls, p0);
        }
        {
          float v[64];
          tc::tmem_ld64(s_row + 64, v);
          mask_half(1, v);
          softmax_pack(v, fac2, nm2, ls, p1);
        }
        tile_sum = ((ls[0].x + ls[0].y) + (ls[1].x + ls[1].y)) + ((ls[2].x + ls[2].y) + (ls[3].x + ls[3].y));
        if (__all_sync(0xffffffffu, tile_sum <= 32768.0f)) {  // false for inf / NaN
          tc::tmem_st32(s_row, p0);
          tc::tmem_st32(s_row + 32, p1);
          done = true;
        }
      }
      if (!done) {
        max_pass();
        tile_sum = exp_pass();
      }
      l_run += tile_sum;
      tc::fence_before();
      mbar_arrive(bar(LY::B_PFULL + qt));
      done_tiles = i + 1;
    }
    // ---- epilogue: this thread's output row, once P . V of the last tile (and, by the order
    // of commits, of every earlier tile) has landed in O
    bool fin = !*abort_flag && done_tiles == n_tiles;
    if (fin && n_tiles > 0)
      fin = wait_or_abort(bar(LY::B_OFULL + qt), (n_tiles - 1) & 1, p.wait_ns, abort_flag);
    if (!__all_sync(0xffffffffu, fin)) {
      *abort_flag = 1;
    } else {
      tc::fence_after();
      const bool sink = p.sinks != nullptr;
      const float inv =
          softmax_out_factor(m_run, l_run, sink, sink ? p.sinks[hq] * 1.4426950408889634f : 0.0f);
      const int64_t ob = (int64_t)b * p.osb + (int64_t)hq * p.osh + (int64_t)l * p.osl;
#pragma unroll
      for (int c = 0; c < DV / 32; ++c) {
        float o_acc[32];
        if (n_tiles > 0) {
          tc::tmem_ld32(o_row + c * 32, o_acc);
        } else {
#pragma unroll
          for (int j2 = 0; j2 < 32; ++j2) o_acc[j2] = 0.0f;
        }
        if (!row_ok) continue;
        if (p.out_dtype == AM_DTYPE_F32) {
          float* o = static_cast<float*>(p.out) + ob + c * 32;
          if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
            for (int d = 0; d < 32; d += 4)
              *reinterpret_cast<float4*>(o + d) =
                  make_float4(o_acc[d] * inv, o_acc[d + 1] * inv, o_acc[d + 2] * inv, o_acc[d + 3] * inv);
          } else {
#pragma unroll
            for (int d = 0; d < 32; ++d) o[d] = o_acc[d] * inv;
          }
        } else {
          const bool bf = p.out_dtype == AM_DTYPE_BF16;
          uint16_t* o = static_cast<uint16_t*>(p.out) + ob + c * 32;
          if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
            for (int d = 0; d < 32; d += 8) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float a = o_acc[d + 2 * e] * inv, c2 = o_acc[d + 2 * e + 1] * inv;
                w[e] = bf ? (static_cast<uint32_t>(f2h<true>(a)) | (static_cast<uint32_t>(f2h<true>(c2)) << 16))
                          : pack_half2(a, c2);
              }
              *reinterpret_cast<uint4*>(o + d) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          } else {
#pragma unroll
            for (int d = 0; d < 32; ++d) o[d] = bf ? f2h<true>(o_acc[d] * inv) : f2h<false>(o_acc[d] * inv);
          }
        }
      }
    }
  }

  // ---- teardown: after an abort, let this CTA's TMA loads and MMAs in flight finish
  // (bounded) before the shared memory and TMEM are released.
  __syncthreads();
  if (*abort_flag) {
    constexpr uint64_t kDrainNs = 100000000ull;
    if (warp == TMA_WARP && lane == 0) {
      for (int jj = max(0, issued_k - NS); jj < issued_k; ++jj)
        mbar_wait_bounded(bar(LY::B_KFULL + jj % NS), (jj / NS) & 1, kDrainNs);
      for (int jj = max(0, issued_v - NS); jj < issued_v; ++jj)
        mbar_wait_bounded(bar(LY::B_VFULL + jj % NS), (jj / NS) & 1, kDrainNs);
    }
    if (warp == MMA_WARP && lane == 0 && mma_issued) {
      tc::commit(bar(LY::B_DRAIN));
      mbar_wait_bounded(bar(LY::B_DRAIN), 0, kDrainNs);
    }
    if (tid == 0) flag_status(p.status, AM_STATUS_TIMEOUT);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                 "r"(LY::TMEM_COLS));
  }
}

// ---------------------------------------------------------------- host side

// Key-tile size and pipeline depths per head-dim pair (shared memory: the query tile, NS K
// stages and NSV V stages must fit one CTA's 227 KB).  The V ring is made the deeper one
// when both cannot grow: V_j can only load once P . V of tile j - NSV has completed, and
// that chain sets the tile period of the largest heads.
template <int DK, int DV>
struct PrefillCfg {
  static constexpr int BN = (DK + DV) > 384 ? 64 : 128;
  template <int K, int V>
  static constexpr bool kFits = PrefillLayout<DK, DV, BN, K, V>::SMEM <= 232448;
  static constexpr int NS = kFits<4, 4> ? 4 : kFits<3, 3> ? 3 : 2;
  static constexpr int NSV = kFits<4, 4> ? 4 : kFits<3, 3> ? 3 : kFits<2, 3> ? 3 : 2;
  using LY = PrefillLayout<DK, DV, BN, NS, NSV>;
};

bool prefill_supported(int k_dim, int v_dim) {
  return (k_dim == 64 && v_dim == 64) || (k_dim == 128 && (v_dim == 128 || v_dim == 64)) ||
         (k_dim == 192 && v_dim == 128) || (k_dim == 256 && v_dim == 256);
}

// Head dims up to 128 take the two-tile kernel (128-key tiles); the others the one-tile kernel.
static bool prefill_two_tiles(int k_dim, int v_dim) { return k_dim <= 128 && v_dim <= 128; }

bool prefill_v_in_kernel(int k_dim, int v_dim) { return k_dim == 192 && v_dim == 128; }

int prefill_key_tile(int k_dim, int v_dim) {
  return prefill_two_tiles(k_dim, v_dim) ? 128 : ((k_dim + v_dim) > 384 ? 64 : 128);
}

// Pipeline depth of the two-tile kernel: as many K/V stages (up to 4) as fit beside the two
// query tiles.
template <int DK, int DV>
struct Prefill2Cfg {
  static constexpr int NS = Prefill2Layout<DK, DV, 4>::SMEM <= 232448   ? 4
                            : Prefill2Layout<DK, DV, 3>::SMEM <= 232448 ? 3
                                                                         : 2;
  using LY = Prefill2Layout<DK, DV, NS>;
};

// cudaFuncSetAttribute is per device: remember, per kernel instantiation, the devices done.
template <typename F>
static cudaError_t prefill_smem_once(F kfn, int bytes, unsigned long long* done_mask) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
  if (bit != 0 && (__atomic_load_n(done_mask, __ATOMIC_ACQUIRE) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit != 0) __atomic_fetch_or(done_mask, bit, __ATOMIC_RELEASE);
  return e;
}

template <int DK, int DV, bool SBF16, bool PAGED>
static cudaError_t launch_stage_t(const DecodeParams& p, int batch, cudaStream_t stream) {
  const int plane_blocks = (p.nw + kStageRows - 1) / kStageRows;
  dim3 grid(p.stage_blocks > 0 ? min(p.stage_blocks, plane_blocks) : plane_blocks, p.hkv, batch);
  prefill_stage_kernel<DK, DV, SBF16, PAGED, kPrefillVInKernel<DK, DV>><<<grid, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

template <int DK, int DV, bool DENSE>
static cudaError_t launch_attn_t(const DecodeParams& p, int batch, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  void (*kfn)(DecodeParams) = nullptr;
  if constexpr (DK <= 128 && DV <= 128) {
    using C = Prefill2Cfg<DK, DV>;
    kfn = prefill2_kernel<DK, DV, C::NS, DENSE>;
    static unsigned long long done = 0;
    cudaError_t e = prefill_smem_once(kfn, C::LY::SMEM, &done);
    if (e != cudaSuccess) return e;
    const int tok_per_cta = 2 * (128 / p.n_rep);
    cfg.gridDim = dim3((p.q_len + tok_per_cta - 1) / tok_per_cta, p.hkv, batch);
    cfg.blockDim = dim3(kTile2Threads);
    cfg.dynamicSmemBytes = C::LY::SMEM;
  } else {
    using C = PrefillCfg<DK, DV>;
    constexpr bool QV4 = kPrefillVInKernel<DK, DV>;
    kfn = prefill_kernel<DK, DV, C::BN, C::NS, C::NSV, DENSE, QV4>;
    static unsigned long long done = 0;
    cudaError_t e = prefill_smem_once(kfn, C::LY::SMEM, &done);
    if (e != cudaSuccess) return e;
    const int tok_per_cta = 128 / p.n_rep;
    cfg.gridDim = dim3((p.q_len + tok_per_cta - 1) / tok_per_cta, p.hkv, batch);
    cfg.blockDim = dim3(PrefillRoles<C::BN, QV4>::THREADS);
    cfg.dynamicSmemBytes = C::LY::SMEM;
  }
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kfn, p);
  if (e == cudaErrorNotSupported || e == cudaErrorInvalidValue) {
    (void)cudaGetLastError();
    kfn<<<cfg.gridDim, cfg.blockDim, cfg.dynamicSmemBytes, stream>>>(p);
    e = cudaGetLastError();
  }
  return e;
}

template <int DK, int DV>
static cudaError_t launch_prefill_dims(const DecodeParams& p0, int batch, bool paged, bool sbf16,
                                       int parts, cudaStream_t stream) {
  DecodeParams p = p0;  // (the attention kernel's V dequantization reads the cache directly)
  p.paged = paged ? 1 : 0;
  p.scale_bf16 = sbf16 ? 1 : 0;
  if (parts & kPrefillStage) {
    cudaError_t e = paged ? (sbf16 ? launch_stage_t<DK, DV, true, true>(p, batch, stream)
                                   : launch_stage_t<DK, DV, false, true>(p, batch, stream))
                          : (sbf16 ? launch_stage_t<DK, DV, true, false>(p, batch, stream)
                                   : launch_stage_t<DK, DV, false, false>(p, batch, stream));
    if (e != cudaSuccess) return e;
  }
  if (!(parts & kPrefillAttend)) return cudaSuccess;
  return p.mask_kind != AM_MASK_NONE ? launch_attn_t<DK, DV, true>(p, batch, stream)
                                     : launch_attn_t<DK, DV, false>(p, batch, stream);
}

cudaError_t launch_prefill(const DecodeParams& p, int batch, bool paged, bool scale_bf16, int parts,
                           cudaStream_t stream) {
  if (p.n_rep < 1 || p.n_rep > 128) return cudaErrorNotSupported;
  if (p.k_dim == 128 && p.v_dim == 128) return launch_prefill_dims<128, 128>(p, batch, paged, scale_bf16, parts, stream);
  if (p.k_dim == 64 && p.v_dim == 64) return launch_prefill_dims<64, 64>(p, batch, paged, scale_bf16, parts, stream);
  if (p.k_dim == 128 && p.v_dim == 64) return launch_prefill_dims<128, 64>(p, batch, paged, scale_bf16, parts, stream);
  if (p.k_dim == 192 && p.v_dim == 128) return launch_prefill_dims<192, 128>(p, batch, paged, scale_bf16, parts, stream);
  if (p.k_dim == 256 && p.v_dim == 256) return launch_prefill_dims<256, 256>(p, batch, paged, scale_bf16, parts, stream);
  return cudaErrorNotSupported;
}

}  // namespace am
