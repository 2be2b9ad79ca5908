// Split-KV flash-decoding attention over a Q4 cache (contiguous or paged), sm_100a.
//
// One CTA = (KV split "chunk", KV head, row group, sequence).  A row group is up to 8
// query rows of one KV head (the n_rep GQA heads times the query positions), so every
// Q4 byte of the chunk is read once for all of them.  4 warps per CTA; each warp streams
// stages of TS tokens (stages w, w+4, ...) through a private ring of NS stages filled by
// 1-D bulk copies, and keeps its own online-softmax state; the 4 warp states are merged
// through shared memory and written as the final output (single chunk), merged with the
// other chunks of the column inside a thread-block cluster through distributed shared
// memory, or written as a partial (m, l, O) that combine_kernel merges across chunks.
//
// Tensor-core use (mma.sync m16n8k16, fp16 in / fp32 accumulate), HBM-bound design:
//  * S = K . Q^T with K as the A operand (16 tokens x 16 dims) and the 8 query rows as N.
//    4-bit codes become fp16 operands with one AND each: the nibble pattern masked into
//    a half's mantissa is the subnormal code * 2^-24 (or code * 2^-20 for the next
//    nibble), so no int->float conversion is needed.  The head-dim order inside each
//    k-step is permuted to match the nibble order (the query fragments carry the same
//    permutation and the 1/16 factor), and each k-step stays inside one 64-dim group so
//    S = sum_g scale_g * (codes_g . q) + bias_g * sum(q_g) applies the group scale and
//    bias to 16x8 results instead of to every element.
//  * O^T = V^T . P with V codes as the A operand (dims x tokens, loaded token-pair
//    interleaved by ldmatrix.trans, one shift and one AND per operand register) and
//    B = P * scale_v (fp16, transposed in registers with movmatrix); the bias term
//    sum_t P * bias_v is accumulated in fp32 on the side.
// The dequantized K/V never exist in memory; per 16 tokens a warp issues DK/16 + DV/16
// MMAs and ~1 ALU op per Q4 element.
//
// Reference semantics followed: mlx_fused_attention.py:69-139 (scale q, q.k^T, mask,
// softmax, P.V; GQA head h -> KV head h / n_rep) and the Metal decode kernel's online
// softmax (mlx_fused_attention.py:320-361).  Accumulation is fp32 throughout.
#include <cfloat>
#include <cstdlib>

#include "am_common.cuh"
#include "am_internal.h"

namespace am {

constexpr int kWarps = 4;
constexpr int kMaxChunk = 8192;            // tokens per CTA chunk (decode_plan never exceeds it)
constexpr int kMaxSplitChunk = 4096;       // chunk cap when the planner splits for parallelism
constexpr int kMaxCluster = 16;            // chunks merged inside one thread-block cluster
constexpr int kMaxBlk = kMaxChunk / 32 + 2;  // block ids a chunk can touch (block_tokens >= 32)
constexpr float kMaskedFinite = -1.0e30f;  // boolean-mask fill (finite: keeps uniform rows)

template <int DK, int DV, int NS, int TS>
struct DecodeLayout {
  static constexpr int NGK = DK / 64, NGV = DV / 64;
  static constexpr int KW = DK / 8, VW = DV / 8;
  static constexpr int KROW = DK / 2, VROW = DV / 2;  // bytes of codes per token row
  // a stage: codes and scales of TS rows, each section as laid out in HBM
  static constexpr int OFF_V = TS * KROW;
  static constexpr int OFF_KS = OFF_V + TS * VROW;
  static constexpr int OFF_KB = OFF_KS + TS * NGK * 2;
  static constexpr int OFF_VS = OFF_KB + TS * NGK * 2;
  static constexpr int OFF_VB = OFF_VS + TS * NGV * 2;
  // K and V code rows of 32, 64 or 128 bytes arrive by swizzled 2-D tensor loads; their
  // tiles then start on 1024-byte boundaries (stages are multiples of 1024 bytes and the
  // V tile offset TS * KROW is one too)
  // (96-byte K rows, Dk = 192, arrive as a 64-byte tile then a 32-byte tile of the same rows)
  static constexpr bool KSPLIT = KROW == 96;
  static constexpr bool SWZ = (KROW == 32 || KROW == 64 || KROW == 128 || KSPLIT) &&
                              (VROW == 32 || VROW == 64 || VROW == 128);
  static constexpr int OFF_K2 = TS * 64;  // KSPLIT: the 32-byte tile of K bytes 64..95
  static constexpr int STAGE_ALIGN = SWZ ? 1024 : 128;
  static constexpr int STAGE = (OFF_VB + TS * NGV * 2 + STAGE_ALIGN - 1) / STAGE_ALIGN * STAGE_ALIGN;
  static_assert(!SWZ || OFF_V % 1024 == 0, "swizzled V tiles start on a 1024-byte boundary");
  static constexpr int RING = NS * STAGE;
  static constexpr int OFF_BAR = kWarps * RING;
  static constexpr int OFF_OK = OFF_BAR + kWarps * NS * 8;
  static constexpr int OFF_BLK = OFF_OK + kWarps * NS * 4;
  // per-column table: int32 [8][4] (hq, l, pos, valid), float [8] prescale, int64 [8]
  // output offset, int64 [8] partial offset, int32 [4] (mask_lo, mask_hi)
  static constexpr int OFF_COL = (OFF_BLK + kMaxBlk * 4 + 15) / 16 * 16;
  static constexpr int SMEM = OFF_COL + 8 * 16 + 8 * 4 + 8 * 8 * 2 + 16;
  // The queries are staged (as fp32 when they fit, else as their 16-bit inputs, plus
  // per-group sums and maxima) in the last stage of warp 0's ring, which no copy touches
  // before the main loop starts.
  // A staged column is padded by 16 bytes, so that the 8 columns' fragment reads (one
  // column per lane group) fall into different banks.
  static constexpr bool Q32 = 8 * (DK + 4) * 4 + 2 * 8 * NGK * 4 <= STAGE;
  static constexpr int QROW = Q32 ? DK + 4 : DK + 8;  // elements per staged column
  static constexpr int OFF_Q = (NS - 1) * STAGE;
  static constexpr int OFF_QS = OFF_Q + 8 * QROW * (Q32 ? 4 : 2);
  static_assert(8 * (DK + 8) * 2 + 2 * 8 * NGK * 4 <= STAGE, "query staging must fit in one stage");
  static_assert((16 + 8 * (DV + 1)) * 4 <= RING, "warp result must fit in its ring");
  static_assert((kWarps * 8 + 24) * 4 <= kMaxBlk * 4, "CTA merge factors must fit in the block-id area");
};

template <int NG, bool BF16>
__device__ __forceinline__ void load_scales(const uint8_t* base, int tok, float (&out)[NG]) {
  const uint16_t* p = reinterpret_cast<const uint16_t*>(base) + tok * NG;
  if constexpr (NG % 2 == 0) {
#pragma unroll
    for (int i = 0; i < NG; i += 2) {
      const uint32_t u = *reinterpret_cast<const uint32_t*>(p + i);
      out[i] = h2f<BF16>(static_cast<uint16_t>(u & 0xffffu));
      out[i + 1] = h2f<BF16>(static_cast<uint16_t>(u >> 16));
    }
  } else {
#pragma unroll
    for (int i = 0; i < NG; ++i) out[i] = h2f<BF16>(p[i]);
  }
}

__device__ __forceinline__ float load_mask(const DecodeParams& p, int b, int hq, int l, int tok) {
  const int64_t idx = (int64_t)b * p.msb + (int64_t)hq * p.msh + (int64_t)l * p.msl +
                      (int64_t)tok * p.msn;
  if (p.mask_kind == AM_MASK_BOOL) return static_cast<const uint8_t*>(p.mask)[idx] ? 1.0f : 0.0f;
  if (p.mask_dtype == AM_DTYPE_F32) return static_cast<const float*>(p.mask)[idx];
  return h2f_rt(static_cast<const uint16_t*>(p.mask)[idx], p.mask_dtype == AM_DTYPE_BF16);
}

// Lazy softmax rescaling: the running max is only raised when a stage's max exceeds it by
// more than 2^3 (log2 units), so P <= 8 and P * scale_v stays well inside fp16.
constexpr float kRescaleSlack = 3.0f;

// Resident CTAs per SM the register allocation aims at: 2 for the largest heads (their
// output accumulators and query fragments alone take ~100 registers a thread), 3 for the
// rest, where shared memory allows no more.  (Without the hint the compiler may settle
// on fewer registers and spill in the streaming loop.)
constexpr int kDecodeMinCtas = 3;
template <int DK, int DV>
constexpr int decode_min_ctas() { return DK + DV >= 512 ? 2 : kDecodeMinCtas; }

template <int DK, int DV, bool SBF16, bool PAGED, int NS, int TS>
__global__ void __launch_bounds__(128, decode_min_ctas<DK, DV>())
    decode_kernel(const __grid_constant__ DecodeParams p) {
  using LY = DecodeLayout<DK, DV, NS, TS>;
  constexpr int NH = TS / 16;  // 16-token MMA tiles per stage
  constexpr int NGK = LY::NGK, NGV = LY::NGV;
  constexpr int KROW = LY::KROW, VROW = LY::VROW;
  constexpr int KSTEPS = DK / 16;
  constexpr int MT = DV / 16;
  // ldmatrix V tiles, except 128-byte rows without the swizzle (8 rows of a tile would share
  // one bank group)
  constexpr bool V_LDSM = VROW <= 64 || LY::SWZ;

  extern __shared__ __align__(1024) uint8_t smem[];

  griddep_launch_dependents();
  griddep_wait();  // everything this kernel reads or writes is ordered after the previous grid

  if constexpr (LY::SWZ) {
    // swizzled tensor loads need 1024-byte aligned tiles: refuse (every CTA alike, so no
    // cluster peer is left waiting) rather than read a shifted pattern
    if (smem_u32(smem) & 1023u) {
      if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
        flag_status(p.status, AM_STATUS_BAD_POSITION);
      return;
    }
  }

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  // Grid: clusters are (chunk, head x row group, sequence) with the chunks of a column
  // along x; otherwise (head x row group, sequence, chunk), so CTAs are dispatched chunk
  // by chunk and the last to run are the highest chunks, each a sequence's shorter tail
  // (long work first, short work last).
  const int rph = p.rows_per_head;
  const int row_groups = (rph + 7) / 8;
  const int hrg = p.cluster ? blockIdx.y : blockIdx.x;
  const int b = p.cluster ? blockIdx.z : blockIdx.y;
  const int chunk = p.cluster ? blockIdx.x : blockIdx.z;
  const int h0 = hrg / row_groups;
  const int rg = hrg % row_groups;

  // The 8 query columns (16-byte vectors) and the sequence's length are independent
  // global loads: issue them together so that their latencies overlap (the stage copies
  // cannot start before the length is known).
  constexpr int QV = 8 * (DK / 8);  // query vectors of the CTA's 8 columns
  constexpr int QPT = (QV + 127) / 128;
  static_assert(QV % 32 == 0, "query vectors fill whole warps");
  uint4 qraw[QPT];
#pragma unroll
  for (int j = 0; j < QPT; ++j) {
    const int i = tid + 128 * j;
    qraw[j] = make_uint4(0u, 0u, 0u, 0u);
    if (QV % 128 == 0 || i < QV) {
      const int c = i / (DK / 8), c8 = i % (DK / 8);
      int rr = rg * 8 + c;
      if (rr >= rph) rr = rph - 1;
      const int l = rr / p.n_rep;
      const int hq = h0 * p.n_rep + rr % p.n_rep;
      qraw[j] = *reinterpret_cast<const uint4*>(p.q + (int64_t)b * p.qsb + (int64_t)hq * p.qsh +
                                                (int64_t)l * p.qsl + c8 * 8);
    }
  }

  const int n = p.kv_len[b];
  const int st = p.kv_start != nullptr ? p.kv_start[b] : 0;
  const bool dense_mask = p.mask_kind != AM_MASK_NONE;
  int lo, hi;
  visible_range(n, st, p.q_len, p.window, dense_mask, TS, lo, hi);
  const int span = max(0, hi - lo);
  const int n_chunks_need = max(1, (span + p.chunk - 1) / p.chunk);
  if (n_chunks_need > p.max_chunks && chunk == 0 && hrg == 0 && threadIdx.x == 0)
    flag_status(p.status, AM_STATUS_BAD_POSITION);  // kv_len beyond the planned max_kv_len
  const int n_chunks_b = min(n_chunks_need, p.max_chunks);
  // A chunk past this sequence's span has no keys.  In cluster mode its CTA still runs to
  // the end (with no stages): every CTA of a cluster takes part in the cluster barriers
  // and in the merge.
  const bool idle = chunk >= n_chunks_b;
  if (idle && !p.cluster) return;
  const int c_lo = lo + chunk * p.chunk;
  const int c_hi = min(c_lo + p.chunk, hi);
  const int n_stages = (!idle && c_hi > c_lo) ? (c_hi - c_lo + TS - 1) / TS : 0;
  const int my_stages = n_stages > warp ? (n_stages - warp + kWarps - 1) / kWarps : 0;

  uint8_t* ring = smem + warp * LY::RING;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LY::OFF_BAR) + warp * NS;
  int32_t* tile_ok = reinterpret_cast<int32_t*>(smem + LY::OFF_OK) + warp * NS;
  int32_t* sblk = reinterpret_cast<int32_t*>(smem + LY::OFF_BLK);
  int32_t* col_i = reinterpret_cast<int32_t*>(smem + LY::OFF_COL);           // [8][4]
  int64_t* col_oo = reinterpret_cast<int64_t*>(smem + LY::OFF_COL + 160);     // [8]
  int64_t* col_wo = reinterpret_cast<int64_t*>(smem + LY::OFF_COL + 224);     // [8]
  int32_t* col_mask = reinterpret_cast<int32_t*>(smem + LY::OFF_COL + 288);   // [2]

  // ------------------------------------------------------------------ barriers, block ids
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < NS; ++s) mbar_init(smem_u32(&bars[s]), 1);
    fence_mbar_init();
  }
  int blk0 = 0;
  if constexpr (PAGED) {
    blk0 = c_lo >> p.bt_shift;
    const int nblk = c_hi > c_lo ? ((c_hi - 1) >> p.bt_shift) - blk0 + 1 : 0;
    for (int i = tid; i < nblk; i += 128) {
      const int bi = blk0 + i;
      int32_t v = bi < p.table_stride ? p.table[(int64_t)b * p.table_stride + bi] : -1;
      if (v < 0 || v >= p.capacity) {
        flag_status(p.status, AM_STATUS_BAD_BLOCK);
        v = -1;
      }
      sblk[i] = v;
    }
  }
  __syncthreads();

  // Lane 0 of each warp fills its ring: a stage = TS rows of K/V codes and scales, six
  // 1-D bulk copies completing on the stage's mbarrier.  A stage never crosses a paged
  // block (block_tokens is a power of two >= TS and stages start on TS boundaries).
  const int64_t head_rows = PAGED ? 0 : ((int64_t)b * p.hkv + h0) * p.capacity;
  auto issue = [&](int k) {
    if (k >= my_stages) return;
    const int s = k % NS;
    const int t0 = c_lo + (warp + kWarps * k) * TS;
    int64_t row0;
    int nrows;
    bool ok = true;
    if constexpr (PAGED) {
      const int32_t v = sblk[(t0 >> p.bt_shift) - blk0];
      ok = v >= 0;
      row0 = ((((int64_t)(ok ? v : 0)) * p.hkv + h0) << p.bt_shift) + (t0 & (p.block_tokens - 1));
      nrows = TS;
    } else {
      row0 = head_rows + t0;
      nrows = min(TS, static_cast<int>(p.capacity - t0));  // capacity and t0 are multiples of 16
    }
    tile_ok[s] = ok ? 1 : 0;
    const uint32_t bar = smem_u32(&bars[s]);
    if (!ok) {
      mbar_arrive(bar);
      return;
    }
    uint8_t* stg = ring + s * LY::STAGE;
    if constexpr (LY::SWZ) {
      // codes: one swizzled box of TS rows each (rows past the array read as zeros)
      mbar_arrive_expect_tx(bar, TS * (KROW + VROW) + nrows * (4 * NGK + 4 * NGV));
      tma_load_2d(smem_u32(stg), &p.tmap_kc, 0, static_cast<int>(row0), bar);
      if constexpr (LY::KSPLIT)
        tma_load_2d(smem_u32(stg + LY::OFF_K2), &p.tmap_kc2, 64, static_cast<int>(row0), bar);
      tma_load_2d(smem_u32(stg + LY::OFF_V), &p.tmap_vc, 0, static_cast<int>(row0), bar);
    } else {
      mbar_arrive_expect_tx(bar, nrows * (KROW + VROW + 4 * NGK + 4 * NGV));
      bulk_g2s(stg, p.kc + row0 * LY::KW, nrows * KROW, bar);
      bulk_g2s(stg + LY::OFF_V, p.vc + row0 * LY::VW, nrows * VROW, bar);
    }
    bulk_g2s(stg + LY::OFF_KS, p.ks + row0 * NGK, nrows * NGK * 2, bar);
    bulk_g2s(stg + LY::OFF_KB, p.kb + row0 * NGK, nrows * NGK * 2, bar);
    bulk_g2s(stg + LY::OFF_VS, p.vs + row0 * NGV, nrows * NGV * 2, bar);
    bulk_g2s(stg + LY::OFF_VB, p.vb + row0 * NGV, nrows * NGV * 2, bar);
  };
  if (lane == 0) {
#pragma unroll
    for (int k = 0; k < NS - 1; ++k) issue(k);
  }

  // ------------------------------------------------------------------ stage queries
  // Column c of the MMA N dimension is query row rg*8 + c of this KV head (row r = l*n_rep
  // + head offset); columns past the head's rows repeat its last row and are never written.
  const bool qbf = p.q_bf16 != 0;
  float* qs32 = reinterpret_cast<float*>(smem + LY::OFF_Q);         // [8][QROW] fp32, or
  uint16_t* qs16 = reinterpret_cast<uint16_t*>(smem + LY::OFF_Q);   // [8][QROW] 16-bit inputs
  float* qsum_s = reinterpret_cast<float*>(smem + LY::OFF_QS);   // [8][NGK]
  float* qmax_s = qsum_s + 8 * NGK;                              // [8][NGK]
  if (tid < 8) {
    const int c = tid;
    int rr = rg * 8 + c;
    const int valid = rr < rph;
    if (!valid) rr = rph - 1;
    const int l = rr / p.n_rep;
    const int hq = h0 * p.n_rep + rr % p.n_rep;
    col_i[c * 4 + 0] = hq;
    col_i[c * 4 + 1] = l;
    col_i[c * 4 + 2] = n - p.q_len + l;
    col_i[c * 4 + 3] = valid;
    col_oo[c] = (int64_t)b * p.osb + (int64_t)hq * p.osh + (int64_t)l * p.osl;
    col_wo[c] = (((int64_t)b * p.hq * p.q_len + (int64_t)hq * p.q_len + l) * p.max_chunks + chunk) *
                (DV + kPartialHead);
    if (c == 0) {
      // keys inside [mask_lo, mask_hi) are visible to every row of the CTA
      const int rows_here = min(8, rph - rg * 8);
      const int pos_min = n - p.q_len + (rg * 8) / p.n_rep;
      const int pos_max = n - p.q_len + (rg * 8 + rows_here - 1) / p.n_rep;
      col_mask[0] = max(st, p.window > 0 ? pos_max - p.window + 1 : 0);
      col_mask[1] = p.causal ? min(n, pos_min + 1) : n;
    }
  }
  // The query vectors to shared memory, with the per (column, 64-dim group) sum and max
  // |q| reduced over the 8 lanes that hold one group (8 consecutive vectors of a column;
  // whole warps take part, as QV is a multiple of 32).
#pragma unroll
  for (int j = 0; j < QPT; ++j) {
    const int i = tid + 128 * j;
    if (QV % 128 == 0 || i < QV) {
      const int c = i / (DK / 8), c8 = i % (DK / 8);
      const uint32_t w[4] = {qraw[j].x, qraw[j].y, qraw[j].z, qraw[j].w};
      float f[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        f[2 * k] = h2f_rt(static_cast<uint16_t>(w[k] & 0xffffu), qbf);
        f[2 * k + 1] = h2f_rt(static_cast<uint16_t>(w[k] >> 16), qbf);
      }
      float sm = 0.0f, mx = 0.0f;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        sm += f[k];
        mx = fmaxf(mx, fabsf(f[k]));
      }
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) {
        sm += __shfl_xor_sync(0xffffffffu, sm, off);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      }
      if ((lane & 7) == 0) {
        qsum_s[c * NGK + c8 / 8] = sm;
        qmax_s[c * NGK + c8 / 8] = mx;
      }
      if constexpr (LY::Q32) {
        *reinterpret_cast<float4*>(qs32 + c * LY::QROW + c8 * 8) = make_float4(f[0], f[1], f[2], f[3]);
        *reinterpret_cast<float4*>(qs32 + c * LY::QROW + c8 * 8 + 4) = make_float4(f[4], f[5], f[6], f[7]);
      } else {
        *reinterpret_cast<uint4*>(qs16 + c * LY::QROW + c8 * 8) = qraw[j];
      }
    }
  }
  __syncthreads();
  // Power-of-two prescale of a column, so that fp16 MMA operands keep full precision:
  // 2^(15 - e) for max |q| in [2^(e-1), 2^e), from its exponent field E (e = E - 126),
  // capped at 2^127 for a tiny or subnormal maximum.
  auto prescale = [&](int c) -> float {
    float m = 0.0f;
#pragma unroll
    for (int G = 0; G < NGK; ++G) m = fmaxf(m, qmax_s[c * NGK + G]);
    if (!(m > 0.0f) || !isfinite(m)) return 1.0f;
    const int E = (__float_as_int(m) >> 23) & 0xff;
    return __int_as_float(min(254, 268 - E) << 23);
  };
  // 8 consecutive query values of column c from dim d (d a multiple of 8)
  auto q8 = [&](int c, int d, float (&f)[8]) {
    if constexpr (LY::Q32) {
      const float4 x = *reinterpret_cast<const float4*>(qs32 + c * LY::QROW + d);
      const float4 y = *reinterpret_cast<const float4*>(qs32 + c * LY::QROW + d + 4);
      f[0] = x.x, f[1] = x.y, f[2] = x.z, f[3] = x.w, f[4] = y.x, f[5] = y.y, f[6] = y.z, f[7] = y.w;
    } else {
      const uint4 r = *reinterpret_cast<const uint4*>(qs16 + c * LY::QROW + d);
      const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        f[2 * k] = h2f_rt(static_cast<uint16_t>(w[k] & 0xffffu), qbf);
        f[2 * k + 1] = h2f_rt(static_cast<uint16_t>(w[k] >> 16), qbf);
      }
    }
  };

  // B fragments of Q for S = K . Q^T.  k-step s = 4G + 2j covers words 8G + 2t + j of
  // column g's slots: nibbles (0, 4) feed k-slots 2t, 2t+1 and nibbles (1, 5) feed 2t+8,
  // 2t+9 (pre-divided by 16).  k-step s + 1 takes bytes 1 and 3 of the words whole: slots
  // 2t, 2t+1 see n2 + 16 n3 (and n6 + 16 n7) with q3 / 16 (q7 / 16), slots 2t+8, 2t+9 see
  // n2 (n6) with q2 - q3 / 16 (q6 - q7 / 16), which sums to n2 q2 + n3 q3 and saves the
  // shift and one mask per operand pair.
  uint32_t qf[KSTEPS][2];
  {
    const float pw = prescale(g);
#pragma unroll
    for (int G = 0; G < NGK; ++G) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int s = 4 * G + 2 * j;
        float x[8];
        q8(g, 8 * (8 * G + 2 * t + j), x);
        qf[s][0] = pack_half2(x[0] * pw, x[4] * pw);
        qf[s][1] = pack_half2(x[1] * pw * 0.0625f, x[5] * pw * 0.0625f);
        const float q3 = x[3] * pw * 0.0625f, q7 = x[7] * pw * 0.0625f;
        qf[s + 1][0] = pack_half2(q3, q7);
        qf[s + 1][1] = pack_half2(fmaf(x[2], pw, -q3), fmaf(x[6], pw, -q7));
      }
    }
  }
  // Per-column (2t, 2t+1) constants.
  // Bias term of the scores, sum_G bias_G[token] * qsum_G[column], as one MMA per 16-token
  // tile: A holds the token's group biases (k = 2G, 2G + 1 both bias_G), B the column's
  // scaled query sums split into a high and a low 16-bit part (k = 2G: high, 2G + 1: low),
  // so the product keeps fp32 accuracy.  Lane (g, t) supplies B for column g, group t.
  uint32_t yb = 0;
  if (t < NGK) {
    const float v = qsum_s[g * NGK + t] * p.scale_log2;
    if constexpr (SBF16) {
      const __nv_bfloat16 hi = __float2bfloat16_rn(v);
      const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
      yb = static_cast<uint32_t>(__bfloat16_as_ushort(hi)) | (static_cast<uint32_t>(__bfloat16_as_ushort(lo)) << 16);
    } else {
      const __half hi = __float2half_rn(v);
      const __half lo = __float2half_rn(v - __half2float(hi));
      yb = static_cast<uint32_t>(__half_as_ushort(hi)) | (static_cast<uint32_t>(__half_as_ushort(lo)) << 16);
    }
  }
  float fac[2];
  int pos_c[2], l_c[2], hq_c[2];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int col = 2 * t + c;
    fac[c] = 16777216.0f / prescale(col) * p.scale_log2;  // 2^24 undoes the subnormal code encoding
    hq_c[c] = col_i[col * 4 + 0];
    l_c[c] = col_i[col * 4 + 1];
    pos_c[c] = col_i[col * 4 + 2];
  }
  // Stages entirely inside [mask_lo, mask_hi) need no per-element masking.
  const int mask_lo = col_mask[0], mask_hi = col_mask[1];
  __syncthreads();  // every warp is done with the staged queries before warp 0 refills that stage

  // ------------------------------------------------------------------ streaming loop
  float o[MT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.0f, 0.0f};
  float vbias[2][NGV];
#pragma unroll
  for (int G = 0; G < NGV; ++G) vbias[0][G] = vbias[1][G] = 0.0f;
  bool aborted = false;
  int consumed = 0;

  for (int k = 0; k < my_stages; ++k) {
    const int s = k % NS;
    if (lane == 0) {
      fence_proxy_async_smem();  // earlier reads of the stage being refilled come first
      issue(k + NS - 1);
    }
    const bool ready = mbar_wait_bounded(smem_u32(&bars[s]), (k / NS) & 1, p.wait_ns);
    if (!__all_sync(0xffffffffu, ready)) {
      aborted = true;
      break;
    }
    consumed = k + 1;
    const uint8_t* stg = ring + s * LY::STAGE;
    const int t0 = c_lo + (warp + kWarps * k) * TS;
    const bool ok = tile_ok[s] != 0;

    // ---- S = K . Q^T, one accumulator set per 16-token tile and 64-dim group ----
    float acc[NH][NGK][4];
#pragma unroll
    for (int hh = 0; hh < NH; ++hh)
#pragma unroll
      for (int G = 0; G < NGK; ++G) acc[hh][G][0] = acc[hh][G][1] = acc[hh][G][2] = acc[hh][G][3] = 0.0f;
#pragma unroll
    for (int G = 0; G < NGK; ++G) {
      uint2 wa[NH], wb[NH];
#pragma unroll
      for (int hh = 0; hh < NH; ++hh) {
        if constexpr (LY::KSPLIT) {
          // bytes 0..63 in the 64-byte tile, 64..95 (group 2) in the 32-byte tile
          if (G < 2) {
            wa[hh] = *reinterpret_cast<const uint2*>(stg + swz_addr<64>(0, hh * 16 + g, G * 32 + t * 8));
            wb[hh] = *reinterpret_cast<const uint2*>(stg + swz_addr<64>(0, hh * 16 + g + 8, G * 32 + t * 8));
          } else {
            wa[hh] = *reinterpret_cast<const uint2*>(stg + LY::OFF_K2 + swz_addr<32>(0, hh * 16 + g, t * 8));
            wb[hh] = *reinterpret_cast<const uint2*>(stg + LY::OFF_K2 + swz_addr<32>(0, hh * 16 + g + 8, t * 8));
          }
        } else if constexpr (LY::SWZ) {
          wa[hh] = *reinterpret_cast<const uint2*>(stg + swz_addr<(LY::SWZ && !LY::KSPLIT) ? KROW : 32>(0, hh * 16 + g, G * 32 + t * 8));
          wb[hh] = *reinterpret_cast<const uint2*>(stg + swz_addr<(LY::SWZ && !LY::KSPLIT) ? KROW : 32>(0, hh * 16 + g + 8, G * 32 + t * 8));
        } else {
          wa[hh] = *reinterpret_cast<const uint2*>(stg + (hh * 16 + g) * KROW + G * 32 + t * 8);
          wb[hh] = *reinterpret_cast<const uint2*>(stg + (hh * 16 + g + 8) * KROW + G * 32 + t * 8);
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int s0 = 4 * G + 2 * j;
#pragma unroll
        for (int hh = 0; hh < NH; ++hh) {
          const uint32_t xa = j ? wa[hh].y : wa[hh].x;
          const uint32_t xb = j ? wb[hh].y : wb[hh].x;
          mma_f16_16816(acc[hh][G], xa & 0x000F000Fu, xb & 0x000F000Fu, xa & 0x00F000F0u,
                        xb & 0x00F000F0u, qf[s0][0], qf[s0][1]);
        }
#pragma unroll
        for (int hh = 0; hh < NH; ++hh) {
          // bytes 1 and 3 into the low bytes of the two halves: n2 + 16 n3, n6 + 16 n7
          const uint32_t xa = __byte_perm(j ? wa[hh].y : wa[hh].x, 0u, 0x4341);
          const uint32_t xb = __byte_perm(j ? wb[hh].y : wb[hh].x, 0u, 0x4341);
          mma_f16_16816(acc[hh][G], xa, xb, xa & 0x000F000Fu, xb & 0x000F000Fu, qf[s0 + 1][0],
                        qf[s0 + 1][1]);
        }
      }
    }
    // scores in log2 units: s2[hh][e] -> token hh*16 + g + 8*(e>>1), column 2t + (e&1)
    float s2[NH][4];
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) {
      float y[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      {
        uint32_t ya0 = 0, ya1 = 0;
        if (t < NGK) {
          const uint16_t* kb = reinterpret_cast<const uint16_t*>(stg + LY::OFF_KB);
          const uint32_t b0 = kb[(hh * 16 + g) * NGK + t], b8 = kb[(hh * 16 + g + 8) * NGK + t];
          ya0 = b0 | (b0 << 16);
          ya1 = b8 | (b8 << 16);
        }
        if constexpr (SBF16) {
          mma_bf16_16816(y, ya0, ya1, 0u, 0u, yb, 0u);
        } else {
          mma_f16_16816(y, ya0, ya1, 0u, 0u, yb, 0u);
        }
      }
#pragma unroll
      for (int tr = 0; tr < 2; ++tr) {
        float sk[NGK];
        load_scales<NGK, SBF16>(stg + LY::OFF_KS, hh * 16 + g + 8 * tr, sk);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int e = 2 * tr + c;
          float x = 0.0f;
#pragma unroll
          for (int G = 0; G < NGK; ++G) x = fmaf(sk[G], acc[hh][G][e], x);
          s2[hh][e] = fmaf(x, fac[c], y[e]);
        }
      }
    }
    // ---- masking (only stages that touch a boundary) ----
    const bool masked_stage = !ok || dense_mask || t0 < mask_lo || t0 + TS > mask_hi;
    if (masked_stage) {
#pragma unroll
      for (int hh = 0; hh < NH; ++hh) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = t0 + hh * 16 + g + 8 * (e >> 1);
          const int c = e & 1;
          bool keep = ok && tok < n && tok >= st;
          if (p.causal && tok > pos_c[c]) keep = false;
          if (p.window > 0 && tok <= pos_c[c] - p.window) keep = false;
          float v = keep ? s2[hh][e] : -INFINITY;
          if (keep && dense_mask) {
            const float mv = load_mask(p, b, hq_c[c], l_c[c], tok);
            if (p.mask_kind == AM_MASK_BOOL) {
              if (mv == 0.0f) v = kMaskedFinite;
            } else {
              v = fmaf(mv, 1.4426950408889634f, v);
            }
          }
          s2[hh][e] = v;
        }
      }
    }
    // ---- online softmax (per column, over the TS tokens of the stage) ----
    float mt[2] = {fmaxf(s2[0][0], s2[0][2]), fmaxf(s2[0][1], s2[0][3])};
#pragma unroll
    for (int hh = 1; hh < NH; ++hh) {
      mt[0] = fmaxf(mt[0], fmaxf(s2[hh][0], s2[hh][2]));
      mt[1] = fmaxf(mt[1], fmaxf(s2[hh][1], s2[hh][3]));
    }
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      mt[c] = fmaxf(mt[c], __shfl_xor_sync(0xffffffffu, mt[c], 4));
      mt[c] = fmaxf(mt[c], __shfl_xor_sync(0xffffffffu, mt[c], 8));
      mt[c] = fmaxf(mt[c], __shfl_xor_sync(0xffffffffu, mt[c], 16));
    }
    // (m_run + slack is -inf while nothing is visible yet, so the first finite max always
    // installs itself)
    if (__any_sync(0xffffffffu, mt[0] > m_run[0] + kRescaleSlack || mt[1] > m_run[1] + kRescaleSlack)) {
      const float mn0 = fmaxf(m_run[0], mt[0]), mn1 = fmaxf(m_run[1], mt[1]);
      const float a0 = m_run[0] == -INFINITY ? 0.0f : ex2(m_run[0] - mn0);
      const float a1 = m_run[1] == -INFINITY ? 0.0f : ex2(m_run[1] - mn1);
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        o[i][0] *= a0;
        o[i][2] *= a0;
        o[i][1] *= a1;
        o[i][3] *= a1;
      }
      l_run[0] *= a0;
      l_run[1] *= a1;
#pragma unroll
      for (int G = 0; G < NGV; ++G) {
        vbias[0][G] *= a0;
        vbias[1][G] *= a1;
      }
      m_run[0] = mn0;
      m_run[1] = mn1;
    }
    const float ms0 = m_run[0] == -INFINITY ? 0.0f : m_run[0];
    const float ms1 = m_run[1] == -INFINITY ? 0.0f : m_run[1];

    // ---- O^T += V^T . (P * scale_v) per 16-token tile ----
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) {
      float pr[4];
      pr[0] = ex2(s2[hh][0] - ms0);
      pr[1] = ex2(s2[hh][1] - ms1);
      pr[2] = ex2(s2[hh][2] - ms0);
      pr[3] = ex2(s2[hh][3] - ms1);
      l_run[0] += pr[0] + pr[2];
      l_run[1] += pr[1] + pr[3];
      // scale / bias of the element's token row (g + 8 tr)
      float bv[2][NGV];
#pragma unroll
      for (int tr = 0; tr < 2; ++tr) load_scales<NGV, SBF16>(stg + LY::OFF_VB, hh * 16 + g + 8 * tr, bv[tr]);
      float bvc[2][2][NGV];  // [tr][column][G]
#pragma unroll
      for (int tr = 0; tr < 2; ++tr)
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int G = 0; G < NGV; ++G) bvc[tr][c][G] = bv[tr][G];
      // B = P * scale_v per 64-dim group, as fp16 pairs (columns 2t, 2t+1) of token rows g
      // and g + 8: fp16 scales multiply the packed P pairs directly (HMUL2); bf16 scales go
      // through fp32
      uint32_t bpk[2][NGV];
      if constexpr (!SBF16) {
        const __half2 p0 = __floats2half2_rn(pr[0], pr[1]), p1 = __floats2half2_rn(pr[2], pr[3]);
#pragma unroll
        for (int tr = 0; tr < 2; ++tr) {
          const uint16_t* sr = reinterpret_cast<const uint16_t*>(stg + LY::OFF_VS) + (hh * 16 + g + 8 * tr) * NGV;
          // an excluded row (p = 0 in both columns) may hold stale shared memory: a zero
          // scale keeps 0 * scale from turning into NaN
          const bool row_live = !masked_stage || pr[2 * tr] > 0.0f || pr[2 * tr + 1] > 0.0f;
#pragma unroll
          for (int G = 0; G < NGV; ++G) {
            const __half sh = row_live ? __ushort_as_half(sr[G]) : __ushort_as_half(0);
            const __half2 prod = __hmul2(tr ? p1 : p0, __half2half2(sh));
            bpk[tr][G] = *reinterpret_cast<const uint32_t*>(&prod);
          }
        }
      } else {
        float sv[2][NGV];
#pragma unroll
        for (int tr = 0; tr < 2; ++tr) load_scales<NGV, SBF16>(stg + LY::OFF_VS, hh * 16 + g + 8 * tr, sv[tr]);
#pragma unroll
        for (int tr = 0; tr < 2; ++tr)
#pragma unroll
          for (int G = 0; G < NGV; ++G) {
            const bool l0 = !masked_stage || pr[2 * tr] > 0.0f, l1 = !masked_stage || pr[2 * tr + 1] > 0.0f;
            bpk[tr][G] = pack_half2(l0 ? pr[2 * tr] * sv[tr][G] : 0.0f, l1 ? pr[2 * tr + 1] * sv[tr][G] : 0.0f);
          }
      }
      if (masked_stage) {
        // rows of excluded keys may hold stale shared memory: zero their bias
#pragma unroll
        for (int tr = 0; tr < 2; ++tr)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const bool live = pr[2 * tr + c] > 0.0f;
#pragma unroll
            for (int G = 0; G < NGV; ++G) bvc[tr][c][G] = live ? bvc[tr][c][G] : 0.0f;
          }
      }
      if constexpr (V_LDSM) {
        // V^T tiles by ldmatrix.trans: matrices (tokens 0-7 | 8-15) x (dims 0-31 | 32-63 of
        // group G); lane (g, t) gets the 4 codes of dims 4g..4g+3 of tokens 2t and 2t+1 in
        // one register, and nibble j of each half is MMA row g's operand for MMA j
        const uint32_t vtile = smem_u32(stg + LY::OFF_V);
        const int vrow = hh * 16 + ((lane >> 4) << 3) + (lane & 7);
        const int vseg = ((lane >> 3) & 1) * 16;
#pragma unroll
        for (int G = 0; G < NGV; ++G) {
          vbias[0][G] = fmaf(pr[0], bvc[0][0][G], fmaf(pr[2], bvc[1][0][G], vbias[0][G]));
          vbias[1][G] = fmaf(pr[1], bvc[0][1][G], fmaf(pr[3], bvc[1][1][G], vbias[1][G]));
          const uint32_t bl = movmatrix_trans(bpk[0][G]);
          const uint32_t bh = movmatrix_trans(bpk[1][G]);
          uint32_t m0, m1, m2, m3;  // (tok 0-7, seg 0) (tok 0-7, seg 1) (tok 8-15, seg 0) (tok 8-15, seg 1)
          const uint32_t va = LY::SWZ ? swz_addr<LY::SWZ ? VROW : 32>(vtile, vrow, G * 32 + vseg)
                                      : vtile + vrow * VROW + G * 32 + vseg;
          ldsm_x4_trans(va, m0, m1, m2, m3);
          // MMA 0 takes byte 0 of each half whole (n0 + 16 n1), MMA 1 its high nibble (16 n1),
          // MMA 2 byte 1 whole (n2 + 16 n3, moved down by a byte permute), MMA 3 its high
          // nibble; the epilogue subtracts the odd accumulators from the even ones
          const uint32_t h0 = __byte_perm(m0, 0u, 0x4341), h1 = __byte_perm(m1, 0u, 0x4341);
          const uint32_t h2 = __byte_perm(m2, 0u, 0x4341), h3 = __byte_perm(m3, 0u, 0x4341);
          mma_f16_16816(o[4 * G + 0], m0 & 0x00FF00FFu, m1 & 0x00FF00FFu, m2 & 0x00FF00FFu,
                        m3 & 0x00FF00FFu, bl, bh);
          mma_f16_16816(o[4 * G + 1], m0 & 0x00F000F0u, m1 & 0x00F000F0u, m2 & 0x00F000F0u,
                        m3 & 0x00F000F0u, bl, bh);
          mma_f16_16816(o[4 * G + 2], h0, h1, h2, h3, bl, bh);
          mma_f16_16816(o[4 * G + 3], h0 & 0x00F000F0u, h1 & 0x00F000F0u, h2 & 0x00F000F0u,
                        h3 & 0x00F000F0u, bl, bh);
        }
      } else {
        // 128-byte V rows (Dv = 256) would put all 8 rows of an ldmatrix tile in one bank
        // group: gather token pairs with byte permutes instead (row-to-row stride 4 lanes)
        const uint8_t* vbase = stg + LY::OFF_V + hh * 16 * VROW;
#pragma unroll
        for (int G = 0; G < NGV; ++G) {
          vbias[0][G] = fmaf(pr[0], bvc[0][0][G], fmaf(pr[2], bvc[1][0][G], vbias[0][G]));
          vbias[1][G] = fmaf(pr[1], bvc[0][1][G], fmaf(pr[3], bvc[1][1][G], vbias[1][G]));
          const uint32_t bl = movmatrix_trans(bpk[0][G]);
          const uint32_t bh = movmatrix_trans(bpk[1][G]);
          const int woff = (8 * G + g) * 4;
          uint32_t v0, v1, v2, v3;
          if constexpr (LY::SWZ) {
            const uint8_t* vt = stg + LY::OFF_V;
            constexpr int VR = LY::SWZ ? VROW : 32;
            v0 = *reinterpret_cast<const uint32_t*>(vt + swz_addr<VR>(0, hh * 16 + 2 * t, woff));
            v1 = *reinterpret_cast<const uint32_t*>(vt + swz_addr<VR>(0, hh * 16 + 2 * t + 1, woff));
            v2 = *reinterpret_cast<const uint32_t*>(vt + swz_addr<VR>(0, hh * 16 + 2 * t + 8, woff));
            v3 = *reinterpret_cast<const uint32_t*>(vt + swz_addr<VR>(0, hh * 16 + 2 * t + 9, woff));
          } else {
            v0 = *reinterpret_cast<const uint32_t*>(vbase + (2 * t) * VROW + woff);
            v1 = *reinterpret_cast<const uint32_t*>(vbase + (2 * t + 1) * VROW + woff);
            v2 = *reinterpret_cast<const uint32_t*>(vbase + (2 * t + 8) * VROW + woff);
            v3 = *reinterpret_cast<const uint32_t*>(vbase + (2 * t + 9) * VROW + woff);
          }
#pragma unroll
          for (int beta = 0; beta < 4; ++beta) {
            const uint32_t sel = beta | ((4 + beta) << 8);
            const uint32_t r01 = __byte_perm(v0, v1, sel);
            const uint32_t r23 = __byte_perm(v2, v3, sel);
            mma_f16_16816(o[4 * G + beta], r01 & 0x000F000Fu, r01 & 0x00F000F0u, r23 & 0x000F000Fu,
                          r23 & 0x00F000F0u, bl, bh);
          }
        }
      }
    }
    __syncwarp();
  }
  if (aborted) {
    if (lane == 0) {
      flag_status(p.status, AM_STATUS_TIMEOUT);
      // give copies already in flight a bounded chance to land before the smem is reused
      for (int k = consumed; k < min(my_stages, consumed + NS); ++k)
        mbar_wait_bounded(smem_u32(&bars[k % NS]), (k / NS) & 1, 100000000ull);
    }
    __syncwarp();
    m_run[0] = m_run[1] = -INFINITY;
    l_run[0] = l_run[1] = 0.0f;
  }

  // ------------------------------------------------------------------ warp reduction
#pragma unroll
  for (int c = 0; c < 2; ++c) {
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l_run[c] += __shfl_xor_sync(0xffffffffu, l_run[c], off);
#pragma unroll
      for (int G = 0; G < NGV; ++G) vbias[c][G] += __shfl_xor_sync(0xffffffffu, vbias[c][G], off);
    }
  }
  // warp result into this warp's (now idle) ring: m[8], l[8], then O[8][DV + 1] (the odd
  // row stride keeps the fragment-order stores at most 2-way bank conflicted)
  constexpr int OS = DV + 1;
  float* wres = reinterpret_cast<float*>(ring);
  if (g == 0) {
    wres[2 * t] = m_run[0];
    wres[2 * t + 1] = m_run[1];
    wres[8 + 2 * t] = l_run[0];
    wres[8 + 2 * t + 1] = l_run[1];
  }
  float* wo = wres + 16;
#pragma unroll
  for (int mt_i = 0; mt_i < MT; ++mt_i) {
    const int G = mt_i / 4, j = mt_i % 4;
    if constexpr (V_LDSM) {
      // tile 4G + j: row g is dim 64G + 4g + j, row g + 8 is dim 64G + 32 + 4g + j; odd j
      // hold the high nibble (code * 2^-20), even j the whole byte (low + 16 * high, so the
      // odd neighbour is subtracted) in units of 2^-24
      const int d = 64 * G + 4 * g + j;
      float ov[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        ov[e] = (j & 1) ? o[mt_i][e] * 1048576.0f : (o[mt_i][e] - o[mt_i + 1][e]) * 16777216.0f;
      wo[(2 * t) * OS + d] = ov[0] + vbias[0][G];
      wo[(2 * t + 1) * OS + d] = ov[1] + vbias[1][G];
      wo[(2 * t) * OS + d + 32] = ov[2] + vbias[0][G];
      wo[(2 * t + 1) * OS + d + 32] = ov[3] + vbias[1][G];
    } else {
      // tile 4G + j: rows g / g + 8 are dims 64G + 8g + 2j / +1 (low / high nibble)
      const int d = 64 * G + 8 * g + 2 * j;
      wo[(2 * t) * OS + d] = fmaf(o[mt_i][0], 16777216.0f, vbias[0][G]);
      wo[(2 * t + 1) * OS + d] = fmaf(o[mt_i][1], 16777216.0f, vbias[1][G]);
      wo[(2 * t) * OS + d + 1] = fmaf(o[mt_i][2], 1048576.0f, vbias[0][G]);
      wo[(2 * t + 1) * OS + d + 1] = fmaf(o[mt_i][3], 1048576.0f, vbias[1][G]);
    }
  }
  __syncthreads();

  // ------------------------------------------------------------------ CTA combine
  // Threads 0..7 merge the warps' (m, l) of one column each into per-warp weights, the CTA
  // max and sum (in the block-id area, free after the loop); then every thread merges
  // output elements.
  float* cf = reinterpret_cast<float*>(smem + LY::OFF_BLK);  // [kWarps][8] weights, M[8], L[8], 1/L[8]
  if (tid < 8) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, reinterpret_cast<const float*>(smem + w * LY::RING)[tid]);
    float L = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float* wr = reinterpret_cast<const float*>(smem + w * LY::RING);
      const float mw = wr[tid];
      const float sc = (mw == -INFINITY) ? 0.0f : ex2(mw - M);
      cf[w * 8 + tid] = sc;
      L = fmaf(wr[8 + tid], sc, L);
    }
    cf[kWarps * 8 + tid] = M;
    cf[kWarps * 8 + 8 + tid] = L;
    const bool sink = p.sinks != nullptr;
    cf[kWarps * 8 + 16 + tid] =
        softmax_out_factor(M, L, sink, sink ? p.sinks[col_i[tid * 4 + 0]] * 1.4426950408889634f : 0.0f);
  }
  __syncthreads();
  float* wres0 = reinterpret_cast<float*>(smem);  // warp 0's result
  const int cols = min(8, rph - rg * 8);          // valid columns are 0 .. cols-1
  for (int i = tid; i < cols * DV; i += 128) {
    const int c = i / DV, d = i % DV;
    float O = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w)
      O = fmaf(reinterpret_cast<const float*>(smem + w * LY::RING)[16 + c * OS + d], cf[w * 8 + c], O);
    if (p.cluster) {
      wres0[16 + c * OS + d] = O;  // in place: only this thread reads or writes element (c, d)
    } else if (n_chunks_b == 1) {
      store_out(p.out, col_oo[c] + d, O * cf[kWarps * 8 + 16 + c], p.out_dtype);
    } else {
      float* slot = p.ws + col_wo[c];
      slot[kPartialHead + d] = O;
      if (d == 0) {
        slot[0] = cf[kWarps * 8 + c];
        slot[1] = cf[kWarps * 8 + 8 + c];
      }
    }
  }
  if (!p.cluster) return;

  // ------------------------------------------------------------------ cluster merge
  // The max_chunks CTAs of this column group form one cluster; each holds its chunk's
  // (M, L) in cf and its O in warp 0's result area.  After the first cluster barrier the
  // CTAs each write an interleaved share of the output elements: a thread reads every
  // chunk's (M, L) of its column and O of its element through distributed shared memory
  // in one round (all loads independent), then merges them.  The second barrier keeps
  // every CTA (and its shared memory) alive until all peers are done reading it.
  cluster_sync_all();
  const int nc = p.max_chunks;
  const uint32_t o_loc = smem_u32(wres0 + 16);
  const bool sink = p.sinks != nullptr;
  for (int i = chunk * 128 + tid; i < cols * DV; i += nc * 128) {
    const int c = i / DV, d = i % DV;
    const uint32_t m_loc = smem_u32(cf + kWarps * 8 + c), l_loc = smem_u32(cf + kWarps * 8 + 8 + c);
    const uint32_t a = o_loc + (c * OS + d) * 4;
    float mj[kMaxCluster], lj[kMaxCluster], xj[kMaxCluster];
#pragma unroll
    for (int j = 0; j < kMaxCluster; ++j) {
      mj[j] = j < nc ? ld_dsmem_f32(dsmem_addr(m_loc, j)) : -INFINITY;
      lj[j] = j < nc ? ld_dsmem_f32(dsmem_addr(l_loc, j)) : 0.0f;
      xj[j] = j < nc ? ld_dsmem_f32(dsmem_addr(a, j)) : 0.0f;
    }
    float M = -INFINITY;
#pragma unroll
    for (int j = 0; j < kMaxCluster; ++j) M = fmaxf(M, mj[j]);
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxCluster; ++j) {
      // a chunk with no visible key (M = -inf) has weight 0 and contributes nothing
      const float w = mj[j] == -INFINITY ? 0.0f : ex2(mj[j] - M);
      L = fmaf(lj[j], w, L);
      O = w != 0.0f ? fmaf(xj[j], w, O) : O;
    }
    const float f = softmax_out_factor(M, L, sink, sink ? p.sinks[col_i[c * 4 + 0]] * 1.4426950408889634f : 0.0f);
    store_out(p.out, col_oo[c] + d, O * f, p.out_dtype);
  }
  cluster_sync_all();
}

// Merge the per-chunk partials of sequences split into more than one chunk.  One warp per
// query row: lanes hold the chunk maxima, the softmax weights are broadcast with shuffles
// and every lane accumulates 16-byte column slices, so all partial loads of a row are
// independent and in flight together.
template <int DV>
__global__ void __launch_bounds__(128) combine_kernel(const DecodeParams p) {
  constexpr int PF = DV + kPartialHead;  // floats per partial record
  constexpr int V4 = DV / 4;             // float4 column slices per row
  constexpr int PER = (V4 + 31) / 32;    // slices per lane
  griddep_launch_dependents();
  griddep_wait();  // the decode grid's partials are complete and visible past this point
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows_total = p.hq * p.q_len;
  const int row = blockIdx.x * 4 + warp;
  const int b = blockIdx.y;
  if (row >= rows_total) return;
  const int n = p.kv_len[b];
  const int st = p.kv_start != nullptr ? p.kv_start[b] : 0;
  int lo, hi;
  visible_range(n, st, p.q_len, p.window, p.mask_kind != AM_MASK_NONE, p.stage_tokens, lo, hi);
  const int span = max(0, hi - lo);
  const int nc = min(max(1, (span + p.chunk - 1) / p.chunk), p.max_chunks);
  if (nc <= 1) return;
  const float* base = p.ws + ((int64_t)b * rows_total + row) * p.max_chunks * PF;

  // the first eight chunks' slices are loaded together with the chunk maxima (independent
  // loads, one round trip)
  float4 x0[8][PER];
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const float4* src = reinterpret_cast<const float4*>(base + (int64_t)u * PF + kPartialHead);
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int v = lane + 32 * k;
      x0[u][k] = (u < nc && (V4 % 32 == 0 || v < V4)) ? src[v] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
  }

  // (max, sum) over this lane's chunks, online, then across the warp
  float m = -INFINITY, l = 0.0f, m_first = -INFINITY;
  for (int c = lane; c < nc; c += 32) {
    const float mc = base[(int64_t)c * PF], lc = base[(int64_t)c * PF + 1];
    if (c == lane) m_first = mc;
    if (mc == -INFINITY) continue;
    const float mn = fmaxf(m, mc);
    l = (m == -INFINITY ? 0.0f : l * ex2(m - mn)) + lc * ex2(mc - mn);
    m = mn;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, m, off);
    const float lo_ = __shfl_xor_sync(0xffffffffu, l, off);
    const float mn = fmaxf(m, mo);
    if (mn != -INFINITY) {
      l = (m == -INFINITY ? 0.0f : l * ex2(m - mn)) + (mo == -INFINITY ? 0.0f : lo_ * ex2(mo - mn));
      m = mn;
    }
  }
  const float M = m;
  float4 acc[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) acc[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int c0 = 0; c0 < nc; c0 += 32) {
    const int c = c0 + lane;
    const float mc = c0 == 0 ? m_first : (c < nc ? base[(int64_t)c * PF] : -INFINITY);
    const float w = (c < nc && mc != -INFINITY) ? ex2(mc - M) : 0.0f;
    const int cnt = min(32, nc - c0);
    // eight chunks' slices are loaded before any is used, so their latencies overlap
    for (int j0 = 0; j0 < cnt; j0 += 8) {
      float4 x[8][PER];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float4* src = reinterpret_cast<const float4*>(base + (int64_t)(c0 + j0 + u) * PF + kPartialHead);
#pragma unroll
        for (int k = 0; k < PER; ++k) {
          const int v = lane + 32 * k;
          if (c0 == 0 && j0 == 0)
            x[u][k] = x0[u][k];  // (loaded above; zeros past nc)
          else
            x[u][k] = (j0 + u < cnt && (V4 % 32 == 0 || v < V4)) ? src[v] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float wj = __shfl_sync(0xffffffffu, w, (j0 + u) & 31);
#pragma unroll
        for (int k = 0; k < PER; ++k) {
          acc[k].x = fmaf(x[u][k].x, wj, acc[k].x);
          acc[k].y = fmaf(x[u][k].y, wj, acc[k].y);
          acc[k].z = fmaf(x[u][k].z, wj, acc[k].z);
          acc[k].w = fmaf(x[u][k].w, wj, acc[k].w);
        }
      }
    }
  }
  const int hq = row / p.q_len, lq = row % p.q_len;
  const bool sink = p.sinks != nullptr;
  const float inv_l = softmax_out_factor(m, l, sink, sink ? p.sinks[hq] * 1.4426950408889634f : 0.0f);
  const int64_t o0 = (int64_t)b * p.osb + (int64_t)hq * p.osh + (int64_t)lq * p.osl;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int v = lane + 32 * k;
    if (V4 % 32 == 0 || v < V4) {
      store_out(p.out, o0 + 4 * v + 0, acc[k].x * inv_l, p.out_dtype);
      store_out(p.out, o0 + 4 * v + 1, acc[k].y * inv_l, p.out_dtype);
      store_out(p.out, o0 + 4 * v + 2, acc[k].z * inv_l, p.out_dtype);
      store_out(p.out, o0 + 4 * v + 3, acc[k].w * inv_l, p.out_dtype);
    }
  }
}

// ---------------------------------------------------------------------- host side

bool decode_supported(int k_dim, int v_dim) {
  return (k_dim == 64 && v_dim == 64) || (k_dim == 128 && v_dim == 128) ||
         (k_dim == 128 && v_dim == 64) || (k_dim == 192 && v_dim == 128) ||
         (k_dim == 256 && v_dim == 256);
}

// Split size (tokens per CTA chunk) for a decode call.  With fewer (sequence, KV head, row
// group) pairs than CTA slots on the device, each pair is split into chunks; the split is
// chosen by a small cost model: waves of CTAs x (fixed per-CTA cost + chunk tokens), where
// the fixed cost (prologue, pipeline fill, CTA merge) is worth ~256 streamed tokens, plus
// the merge of split chunks, with chunks of at most 4096 tokens.  With at least a full
// wave of pairs, chunks are as long as allowed (8192 tokens: fewer CTA prologues and
// partials to merge; measured 8% faster than 2048-token chunks on 256 agents).
//
// A chunk is costed between its tokens and whole rounds of 4 stages (the CTA's warps
// stream stages in parallel).  Split chunks merge either through the workspace and a
// second launch (combine_kernel, ~320 tokens' worth of latency) or, when every column's
// chunks form one thread-block cluster and all clusters are resident at once, inside the
// cluster (*cluster = 1: ~64 tokens' worth plus 12 per chunk read, no workspace).  Cluster CTAs are held until the whole cluster is done,
// so a grid of several waves keeps the workspace merge.
// Fixed per-CTA cost of a decode chunk in the split planner, in streamed tokens' worth.
constexpr int kPlanFixedTokens = 256;

void decode_plan(int batch, int n_kv_heads, int row_groups, int span, int ctas_per_sm, int k_dim,
                 int v_dim, int* chunk, int* n_chunks, int* cluster) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    sms = 148;
    (void)cudaGetLastError();  // clear: this query must not poison a later launch check
  }
  const int64_t pairs = (int64_t)batch * n_kv_heads * row_groups;
  const int64_t slots = (int64_t)sms * (ctas_per_sm > 0 ? ctas_per_sm : 1);
  const int64_t sp = span > 0 ? span : 1;
  auto chunk_for = [&](int64_t n_split, int64_t cap) {
    int64_t c = (sp + n_split - 1) / n_split;
    c = (c + 63) / 64 * 64;
    return c < 128 ? (int64_t)128 : (c > cap ? cap : c);
  };
  constexpr int64_t kFixed = kPlanFixedTokens, kCombine = 320, kClusterMerge = 64, kClusterPerChunk = 12;
  // the 4 warps of a CTA stream stages in parallel, so a partial round of 4 stages costs
  // about half a round more than its tokens (measured: 2-stage chunks take most of a
  // 4-stage chunk's time)
  const int64_t round_tokens = (int64_t)kWarps * decode_stage_tokens(k_dim, v_dim);
  auto chunk_cost = [&](int64_t c) {
    return kFixed + (c + (c + round_tokens - 1) / round_tokens * round_tokens) / 2;
  };
  const int max_cluster = pairs < slots ? decode_max_cluster(k_dim, v_dim) : 0;
  // cluster merge possible for nch chunks per column: all pairs' clusters resident at once
  auto cluster_ok = [&](int64_t nch) {
    return nch >= 2 && nch <= max_cluster && pairs <= decode_active_clusters(k_dim, v_dim, (int)nch);
  };
  int64_t best_c = chunk_for(1, kMaxChunk);
  bool best_cluster = false;
  if (pairs < slots) {
    int64_t best_cost = -1;
    const int64_t max_split = (4 * slots + pairs - 1) / pairs;
    for (int64_t n = 1; n <= max_split; ++n) {
      const int64_t c = chunk_for(n, kMaxSplitChunk);
      const int64_t nch = (sp + c - 1) / c;
      const int64_t ctas = pairs * nch;
      int64_t cost = ((ctas + slots - 1) / slots) * chunk_cost(c) + (nch > 1 ? kCombine : 0);
      bool cl = false;
      // the in-cluster merge reads every chunk's partial: its cost grows with the cluster
      const int64_t cl_cost = chunk_cost(c) + kClusterMerge + kClusterPerChunk * nch;
      if (cluster_ok(nch) && cl_cost < cost) {
        cost = cl_cost;
        cl = true;
      }
      if (best_cost < 0 || cost < best_cost) {
        best_cost = cost;
        best_c = c;
        best_cluster = cl;
      }
    }
  }
  *chunk = static_cast<int>(best_c);
  *n_chunks = static_cast<int>((sp + best_c - 1) / best_c);
  if (*n_chunks < 1) *n_chunks = 1;
  *cluster = (best_cluster && *n_chunks >= 2) ? 1 : 0;
}

// Launch with programmatic stream serialization: the grid may become resident while the
// previous kernel in the stream finishes (it waits in griddep_wait() before touching
// memory).  Streams or drivers that refuse the attribute get a plain launch.
// cluster_x > 1 launches thread-block clusters of (cluster_x, 1, 1) CTAs.
template <typename... Args>
static cudaError_t launch_pdl(void (*kfn)(Args...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, const DecodeParams& p, int cluster_x = 1) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x > 1 ? cluster_x : 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  const bool clustered = cluster_x > 1;
  cfg.attrs = clustered ? attr : attr + 1;
  cfg.numAttrs = clustered ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kfn, p);
  if (e == cudaErrorNotSupported || e == cudaErrorInvalidValue) {
    (void)cudaGetLastError();
    if (clustered) {
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      e = cudaLaunchKernelEx(&cfg, kfn, p);
    } else {
      kfn<<<grid, block, smem, stream>>>(p);
      e = cudaGetLastError();
    }
  }
  return e;
}

// cudaFuncSetAttribute is per device: remember, per kernel instantiation, the devices done.
template <typename F>
static cudaError_t set_smem_once(F kfn, int bytes, unsigned long long* done_mask) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
  if (bit != 0 && (__atomic_load_n(done_mask, __ATOMIC_ACQUIRE) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit != 0) __atomic_fetch_or(done_mask, bit, __ATOMIC_RELEASE);
  return e;
}

// Largest stage (bytes) that gets a 3-stage ring per warp.
constexpr int kDecodeNs3MaxStage = 6144;

// Stage geometry of an instantiation: 64-token stages when a token row of K and V is
// small (Dk + Dv <= 256), so the per-stage work (copy issue, barrier wait, softmax max)
// is spread over more tokens; 32-token stages for larger heads.  Three stages per warp
// when a stage is at most 6 KB, else two.  (Head dims 256/256 measured no faster with
// three 9 KB stages: at 2 CTAs per SM their stage time is set by instruction issue, not
// by the copies in flight.)
template <int DK, int DV>
struct DecodeCfg {
  static constexpr int TS = DK + DV <= 256 ? 64 : 32;
  static constexpr int NS = DecodeLayout<DK, DV, 3, TS>::STAGE <= kDecodeNs3MaxStage ? 3 : 2;
  using LY = DecodeLayout<DK, DV, NS, TS>;
};

// Clusters of more than 8 CTAs are opt-in per kernel (and per device).
template <typename F>
static cudaError_t allow_large_clusters_once(F kfn, unsigned long long* done_mask) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
  if (bit != 0 && (__atomic_load_n(done_mask, __ATOMIC_ACQUIRE) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kfn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess && bit != 0) __atomic_fetch_or(done_mask, bit, __ATOMIC_RELEASE);
  return e;
}

template <int DK, int DV, bool SBF16, bool PAGED>
static cudaError_t launch_decode_t(const DecodeParams& p, int batch, int row_groups,
                                   cudaStream_t stream) {
  using CF = DecodeCfg<DK, DV>;
  using LY = typename CF::LY;
  auto kfn = decode_kernel<DK, DV, SBF16, PAGED, CF::NS, CF::TS>;
  static unsigned long long smem_done = 0, cluster_done = 0;
  cudaError_t e = set_smem_once(kfn, LY::SMEM, &smem_done);
  if (e != cudaSuccess) return e;
  if (p.cluster) {
    const dim3 grid(p.max_chunks, p.hkv * row_groups, batch);
    if (p.max_chunks > 8) {
      e = allow_large_clusters_once(kfn, &cluster_done);
      if (e != cudaSuccess) return e;
    }
    return launch_pdl(kfn, grid, dim3(128), LY::SMEM, stream, p, p.max_chunks);
  }
  e = launch_pdl(kfn, dim3(p.hkv * row_groups, batch, p.max_chunks), dim3(128), LY::SMEM, stream, p);
  if (e != cudaSuccess) return e;
  if (p.max_chunks > 1) {
    const int rows_total = p.hq * p.q_len;
    e = launch_pdl(combine_kernel<DV>, dim3((rows_total + 3) / 4, batch), dim3(128), 0, stream, p);
  }
  return e;
}

// Resident decode CTAs per SM for a head-dim pair (the paged fp16-scale instantiation
// stands for all four: same registers and shared memory), cached per device.
template <int DK, int DV>
static int ctas_per_sm_t() {
  using CF = DecodeCfg<DK, DV>;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return 1;
  }
  if (dev >= 0 && dev < 64) {
    const int v = __atomic_load_n(&cache[dev], __ATOMIC_ACQUIRE);
    if (v > 0) return v;
  }
  auto kfn = decode_kernel<DK, DV, false, true, CF::NS, CF::TS>;
  static unsigned long long smem_done = 0;
  int n = 0;
  if (set_smem_once(kfn, CF::LY::SMEM, &smem_done) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kfn, 128, CF::LY::SMEM) != cudaSuccess ||
      n < 1) {
    (void)cudaGetLastError();
    return 1;
  }
  if (dev >= 0 && dev < 64) __atomic_store_n(&cache[dev], n, __ATOMIC_RELEASE);
  return n;
}

int decode_ctas_per_sm(int k_dim, int v_dim) {
  if (k_dim == 64 && v_dim == 64) return ctas_per_sm_t<64, 64>();
  if (k_dim == 128 && v_dim == 128) return ctas_per_sm_t<128, 128>();
  if (k_dim == 128 && v_dim == 64) return ctas_per_sm_t<128, 64>();
  if (k_dim == 192 && v_dim == 128) return ctas_per_sm_t<192, 128>();
  if (k_dim == 256 && v_dim == 256) return ctas_per_sm_t<256, 256>();
  return 1;
}

int decode_stage_tokens(int k_dim, int v_dim) { return k_dim + v_dim <= 256 ? 64 : 32; }

// Resident clusters of `size` decode CTAs (2 .. kMaxCluster) for a head-dim pair on the
// current device, cached per device and size; 0 when such a cluster cannot be scheduled.
template <int DK, int DV>
static int active_clusters_t(int size) {
  using CF = DecodeCfg<DK, DV>;
  static int cache[64][kMaxCluster + 1] = {};  // 0: not queried, -1: none
  if (size < 2 || size > kMaxCluster) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  if (dev >= 0 && dev < 64) {
    const int v = __atomic_load_n(&cache[dev][size], __ATOMIC_ACQUIRE);
    if (v != 0) return v > 0 ? v : 0;
  }
  auto kfn = decode_kernel<DK, DV, false, true, CF::NS, CF::TS>;
  static unsigned long long smem_done = 0, cluster_done = 0;
  int n = 0;
  bool ok = set_smem_once(kfn, CF::LY::SMEM, &smem_done) == cudaSuccess &&
            (size <= 8 || allow_large_clusters_once(kfn, &cluster_done) == cudaSuccess);
  if (ok) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(size, 1, 1);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = CF::LY::SMEM;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = size;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ok = cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) == cudaSuccess;
  }
  (void)cudaGetLastError();
  if (!ok || n < 1) n = -1;
  if (dev >= 0 && dev < 64) __atomic_store_n(&cache[dev][size], n, __ATOMIC_RELEASE);
  return n > 0 ? n : 0;
}

int decode_active_clusters(int k_dim, int v_dim, int size) {
  if (k_dim == 64 && v_dim == 64) return active_clusters_t<64, 64>(size);
  if (k_dim == 128 && v_dim == 128) return active_clusters_t<128, 128>(size);
  if (k_dim == 128 && v_dim == 64) return active_clusters_t<128, 64>(size);
  if (k_dim == 192 && v_dim == 128) return active_clusters_t<192, 128>(size);
  if (k_dim == 256 && v_dim == 256) return active_clusters_t<256, 256>(size);
  return 0;
}

// Largest cluster of decode CTAs (up to kMaxCluster) that the device can schedule for a
// head-dim pair; 0 when clusters are unavailable.  AM_Q4_DECODE_MAX_CLUSTER (read on every
// call) lowers the cap: 0 or 1 turns cluster merging off, so split chunks go through the
// workspace and combine_kernel.
int decode_max_cluster(int k_dim, int v_dim) {
  int m = 0;
  for (int size : {kMaxCluster, 8, 4, 2}) {
    if (decode_active_clusters(k_dim, v_dim, size) > 0) {
      m = size;
      break;
    }
  }
  if (const char* env = getenv("AM_Q4_DECODE_MAX_CLUSTER")) {
    const int cap = atoi(env);
    if (cap < m) m = cap < 2 ? 0 : cap;
  }
  return m;
}

template <int DK, int DV>
static cudaError_t launch_decode_d(const DecodeParams& p, int batch, int row_groups, bool paged,
                                   bool sbf16, cudaStream_t stream) {
  if (paged) {
    return sbf16 ? launch_decode_t<DK, DV, true, true>(p, batch, row_groups, stream)
                 : launch_decode_t<DK, DV, false, true>(p, batch, row_groups, stream);
  }
  return sbf16 ? launch_decode_t<DK, DV, true, false>(p, batch, row_groups, stream)
               : launch_decode_t<DK, DV, false, false>(p, batch, row_groups, stream);
}

cudaError_t launch_decode(const DecodeParams& p, int batch, int row_groups, bool paged,
                          bool scale_bf16, cudaStream_t stream) {
  const int dk = p.k_dim, dv = p.v_dim;
  if (p.stage_tokens != decode_stage_tokens(dk, dv)) return cudaErrorInvalidValue;
  if (dk == 64 && dv == 64) return launch_decode_d<64, 64>(p, batch, row_groups, paged, scale_bf16, stream);
  if (dk == 128 && dv == 128) return launch_decode_d<128, 128>(p, batch, row_groups, paged, scale_bf16, stream);
  if (dk == 128 && dv == 64) return launch_decode_d<128, 64>(p, batch, row_groups, paged, scale_bf16, stream);
  if (dk == 192 && dv == 128) return launch_decode_d<192, 128>(p, batch, row_groups, paged, scale_bf16, stream);
  if (dk == 256 && dv == 256) return launch_decode_d<256, 256>(p, batch, row_groups, paged, scale_bf16, stream);
  return cudaErrorNotSupported;
}

}  // namespace am
