// Chunked-prefill attention over a Q4 cache on 5th-generation tensor cores (tcgen05).
//
// One CTA = 128 query rows of one KV head of one sequence.  Rows are (token, GQA head)
// pairs, token-major: 128 / n_rep query tokens times the n_rep heads that share the KV
// head, so each dequantized K/V tile feeds all of them.  384 threads, warp-specialised:
//   * producer warps 8-11 dequantize the Q4 K and V rows of 128-key tile j (one token per
//     thread, raw rows prefetched one tile ahead; fp16 magic-number dequantisation) into
//     fp16 operand tiles in shared memory (128-byte swizzle; K K-major, V MN-major; three
//     buffers), then one producer thread issues S_j = Q . K_j^T (tcgen05.mma kind::f16,
//     M=128, N=128, K=16 steps) into TMEM S[j%2];
//   * softmax warps 0-7: warp w owns TMEM lanes 32(w%4) .. +31 (one query row per thread)
//     and key columns 64(w/4) .. +63 of each tile; tcgen05.ld of its half row, row maxima
//     exchanged with the partner warp through shared memory, fp32 online softmax, P as
//     fp16 pairs stored back over the warp's own S columns (tcgen05.st); O rows rescaled in
//     TMEM only when the running max moves by more than 2^8.  Once all 256 softmax threads
//     have written P (an mbarrier), lane 0 of warp 0 issues O += P_j . V_j with A = P read
//     from TMEM (accumulating after the first tile); its commit frees the S buffer.
// mbarriers (MMA commits and thread arrivals) chain the stages so the dequantisation of
// tile j+1, the MMAs of tile j and the softmax of tile j overlap.  TMEM: S x2 + O (512
// columns, one CTA per SM).  Operands are fp16 for every query dtype: bf16 queries are
// rescaled per row by a power of two so the conversion is exact.  Every mbarrier wait is
// bounded (2 s of %globaltimer); on timeout the kernel flags AM_STATUS_TIMEOUT, stops
// issuing work, frees its TMEM and returns.
//
// Reference semantics: the compiled quantized SDPA (mlx_fused_attention.py:69-139) as
// used by chunked prefill (batch_engine.py:339-456): the chunk's own K/V are already in
// the Q4 cache (quantize-on-append runs first, mlx_quantized_extensions.py:273-298) and
// query l of the chunk sits at position kv_len - q_len + l.
#include "am_common.cuh"
#include "am_internal.h"

namespace am {

namespace tc {

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
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
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
#undef AM_R8

// Warp loads 32 lanes x 64 consecutive fp32 columns of TMEM in one instruction.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
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
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// Warp loads 32 lanes x 128 consecutive fp32 columns of TMEM in one instruction (a whole
// S row per thread: one TMEM round trip per tile).
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, float (&v)[128]) {
  uint32_t r[128];
#define AM_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), \
                 "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 {"
      "%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,"
      "%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,"
      "%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,"
      "%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,"
      "%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%128];\n"
      : AM_R8(0), AM_R8(8), AM_R8(16), AM_R8(24), AM_R8(32), AM_R8(40), AM_R8(48), AM_R8(56),
        AM_R8(64), AM_R8(72), AM_R8(80), AM_R8(88), AM_R8(96), AM_R8(104), AM_R8(112), AM_R8(120)
      : "r"(taddr));
#undef AM_R8
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 128; ++i) v[i] = __uint_as_float(r[i]);
}

// Warp stores 32 lanes x 32 consecutive fp32 columns of TMEM (thread i -> lane base+i).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]),
      "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]),
      "f"(v[16]), "f"(v[17]), "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]),
      "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}

// Warp stores 32 lanes x 32 consecutive 32-bit columns of TMEM (thread i -> lane base+i).
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t (&v)[32]) {
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

// Byte offset inside a 1024-byte-aligned 128B-swizzled region.
__device__ __forceinline__ uint32_t swz(uint32_t off) { return off ^ (((off >> 7) & 7u) << 4); }

}  // namespace tc

template <int D>
struct PrefillLayout {
  static constexpr int TILE = 128 * 128 * 2;  // 128 rows x up to 128 fp16 (Q, K, V tiles)
  static constexpr int NKV = 3;                // K/V tile buffers (P lives in TMEM)
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + TILE;        // NKV K buffers
  static constexpr int OFF_V = OFF_K + NKV * TILE;  // NKV V buffers
  static constexpr int OFF_QF = OFF_V + NKV * TILE;  // per-row query factor (128 floats)
  static constexpr int OFF_RX = OFF_QF + 128 * 4;   // per-row exchange between column halves [2][128]
  static constexpr int OFF_BAR = OFF_RX + 2 * 128 * 4;
  static constexpr int SMEM = OFF_BAR + 128 + 1024;  // barriers + slack for 1024-byte alignment
  static constexpr uint32_t TMEM_COLS = 512;     // S x2 (256) + O (D, accumulated over tiles)
  static_assert(D <= 128, "tiles sized for D <= 128");
  static_assert(SMEM <= 232448, "dynamic shared memory of one CTA");
};

// Multiply this thread's TMEM row of the O accumulator (D columns at taddr) by f.
template <int D>
__device__ __forceinline__ void rescale_o(uint32_t taddr, float f) {
#pragma unroll 1
  for (int c = 0; c < D / 32; ++c) {
    float v[32];
    tc::tmem_ld32(taddr + c * 32, v);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] *= f;
    tc::tmem_st32(taddr + c * 32, v);
  }
}

// Lazy rescaling: a row's running max is raised only when a tile's max exceeds it by more
// than 2^8 (log2 units), so P <= 256 (exact range for the fp16 P operand) and the O
// accumulator in TMEM is rescaled rarely.
constexpr float kPrefillRescaleSlack = 8.0f;

// Operand tiles hold the 8 head dims of every 16-byte chunk in the order the dequantiser
// produces them, kPerm8[p] = head dim of position p: the Q4 word of 8 nibbles n0..n7 (dims
// 0..7) becomes the half pairs (n0, n4) (n1, n5) (n2, n6) (n3, n7) with one mask each.  Q
// carries the same order (so S = Q . K^T is unchanged) and O's columns come out in it, so
// the epilogue puts them back.
__device__ __forceinline__ constexpr int perm8(int p) { return (p & 1) ? (p >> 1) + 4 : (p >> 1); }

// 8 Q4 codes of one word -> 8 fp16 values code * s + b in perm8 order (16 bytes).  A code
// OR-ed into the mantissa of 1024.0 is the fp16 value 1024 + code; subtracting 1024 leaves
// the code exactly, then one fp16 FMA applies scale and bias with a single rounding.
__device__ __forceinline__ uint4 dequant8(uint32_t w, __half2 s2, __half2 b2) {
  const __half2 k1024 = __half2half2(__ushort_as_half(0x6400));
  uint32_t out[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint32_t x = ((w >> (4 * e)) & 0x000F000Fu) | 0x64006400u;
    __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&x), k1024);
    h = __hfma2(h, s2, b2);
    out[e] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

template <bool BF16>
__device__ __forceinline__ __half2 scale_h2(uint16_t bits) {
  if constexpr (BF16) {
    return __half2half2(__float2half_rn(h2f<true>(bits)));
  } else {
    return __half2half2(__ushort_as_half(bits));
  }
}

// 12 warps: softmax warps 0-7 (warp w: S rows 32 (w % 4) .. +31, key columns 64 (w / 4)
// .. +63 -- TMEM lane quarter w % 4 is the only one warp w may access), producer warps 8-11.
constexpr int kPrefillThreads = 384;
constexpr int kSoftmaxThreads = 256;

// mbarrier slots (8 bytes each) inside OFF_BAR
enum { B_SFULL = 0, B_SFREE = 2, B_OFULL = 4, B_KVFREE = 5, B_PFULL = 8, B_COUNT = 9 };

// Named barrier over one 128-thread warp group that also ORs a flag across it: every
// thread gets the same answer, so a group leaves its loop together even if the shared
// abort flag changes while its threads read it.
__device__ __forceinline__ bool group_bar_any(int id, bool v, int count = 128) {
  uint32_t r;
  asm volatile(
      "{\n.reg .pred p, q;\nsetp.ne.u32 p, %1, 0;\nbar.red.or.pred q, %2, %3, p;\n"
      "selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void named_bar_producers() {
  asm volatile("bar.sync 1, 128;\n" ::: "memory");
}

template <int D, bool SBF16, bool PAGED, bool DENSE>
__global__ void __launch_bounds__(kPrefillThreads, 1) prefill_kernel(const DecodeParams p) {
  using LY = PrefillLayout<D>;
  constexpr int NG = D / 64;
  constexpr int KSTEPS = D / 16;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_addr & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  const uint32_t s_base = raw_addr + pad;
  const uint32_t sQ = s_base + LY::OFF_Q, sK = s_base + LY::OFF_K, sV = s_base + LY::OFF_V;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LY::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + LY::OFF_BAR + B_COUNT * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + LY::OFF_BAR + B_COUNT * 8 + 4);
  float* sqf = reinterpret_cast<float*>(smem + LY::OFF_QF);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const bool producer = warp >= 8;
  // Grid (KV head, sequence, query tile) with the query tile slowest and reversed: under
  // the causal mask later query tiles see more keys, so the heaviest CTAs are dispatched
  // first and the lightest fill the last wave.
  const int h = blockIdx.x, b = blockIdx.y;
  const int n_rep = p.n_rep;
  const int tok_per_cta = 128 / n_rep;
  const int l0 = (gridDim.z - 1 - blockIdx.z) * tok_per_cta;
  const int l_last = min(l0 + tok_per_cta, p.q_len) - 1;

  const int n = p.kv_len[b];
  const int st = p.kv_start != nullptr ? p.kv_start[b] : 0;
  const int pos_min = n - p.q_len + l0, pos_max = n - p.q_len + l_last;
  int lo = 0, hi = n;
  if (!DENSE) {
    lo = max(st, 0);
    if (p.window > 0) lo = max(lo, pos_min - p.window + 1);
  }
  if (p.causal) hi = min(hi, pos_max + 1);
  const int n_tiles = hi > lo ? (hi - lo + 127) / 128 : 0;

  // ---- setup
  if (tid == 0) {
    mbar_init(bar(B_SFULL), 1);
    mbar_init(bar(B_SFULL + 1), 1);
    mbar_init(bar(B_SFREE), 1);  // P . V of the tile done: S (which then holds P) is free
    mbar_init(bar(B_SFREE + 1), 1);
    mbar_init(bar(B_OFULL), 1);
    mbar_init(bar(B_PFULL), kSoftmaxThreads);
    for (int b2 = 0; b2 < LY::NKV; ++b2) mbar_init(bar(B_KVFREE + b2), 1);
    fence_mbar_init();
    *abort_flag = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(LY::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  if (producer) {
    // query row r = tid - 256 -> fp16 with a power-of-two prescale (exact for fp16 / bf16)
    const int r = tid - kSoftmaxThreads;
    const int rl = r / n_rep;
    const bool row_ok = r < tok_per_cta * n_rep && l0 + rl < p.q_len;
    const int l = l0 + (row_ok ? rl : 0);
    const int hq = h * n_rep + r % n_rep;
    const uint16_t* qrow = p.q + (int64_t)b * p.qsb + (int64_t)hq * p.qsh + (int64_t)l * p.qsl;
    float amax = 0.0f;
    if (row_ok) {
#pragma unroll 1
      for (int c = 0; c < D / 8; ++c) {
        const uint4 raw = *reinterpret_cast<const uint4*>(qrow + c * 8);
        const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          amax = fmaxf(amax, fabsf(h2f_rt(u[i] & 0xffffu, p.q_bf16)));
          amax = fmaxf(amax, fabsf(h2f_rt(u[i] >> 16, p.q_bf16)));
        }
      }
    }
    float pw = 1.0f;
    if (amax > 0.0f && isfinite(amax)) {
      int e;
      frexpf(amax, &e);
      pw = ldexpf(1.0f, 15 - e);
    }
    sqf[r] = p.scale_log2 / pw;
#pragma unroll 1
    for (int c = 0; c < D / 8; ++c) {
      uint4 outv = make_uint4(0, 0, 0, 0);
      if (row_ok) {
        const uint4 raw = *reinterpret_cast<const uint4*>(qrow + c * 8);
        const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
        float qv[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          qv[2 * i] = h2f_rt(u[i] & 0xffffu, p.q_bf16) * pw;
          qv[2 * i + 1] = h2f_rt(u[i] >> 16, p.q_bf16) * pw;
        }
        uint32_t o4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) o4[i] = pack_half2(qv[perm8(2 * i)], qv[perm8(2 * i + 1)]);
        outv = make_uint4(o4[0], o4[1], o4[2], o4[3]);
      }
      const uint32_t off = (c / 8) * (128 * 128) + r * 128 + (c % 8) * 16;
      *reinterpret_cast<uint4*>(smem + LY::OFF_Q + tc::swz(off)) = outv;
    }
  }
  tc::fence_proxy_async();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr uint32_t ID_S = tc::idesc(128, 128, false);
  constexpr uint32_t ID_O = tc::idesc(128, D, true);

  if (producer) {
    // ================================================================ producer warps
    const int r = tid - kSoftmaxThreads;  // token row of each K/V tile this thread dequantizes
    // Raw Q4 data of this thread's row of a tile, loaded one tile ahead so the global
    // loads of tile j+1 are in flight while tile j is dequantized.
    struct RawRow {
      uint4 k[NG * 2], v[NG * 2];
      uint16_t ks[NG], kb[NG], vs[NG], vb[NG];
      bool valid;
    };
    auto load_raw = [&](int j, RawRow& R) {
      const int tok = lo + j * 128 + r;
      R.valid = tok < n && tok >= 0;
      int64_t row = 0;
      if (R.valid) {
        if constexpr (PAGED) {
          const int bi = tok / p.block_tokens;
          const int32_t blk = bi < p.table_stride ? p.table[(int64_t)b * p.table_stride + bi] : -1;
          if (blk < 0 || blk >= p.capacity) {
            R.valid = false;
            flag_status(p.status, AM_STATUS_BAD_BLOCK);
          } else {
            row = ((int64_t)blk * p.hkv + h) * p.block_tokens + tok % p.block_tokens;
          }
        } else {
          row = ((int64_t)b * p.hkv + h) * p.capacity + tok;
        }
      }
      const uint4* kc = reinterpret_cast<const uint4*>(p.kc + row * (D / 8));
      const uint4* vc = reinterpret_cast<const uint4*>(p.vc + row * (D / 8));
#pragma unroll
      for (int i = 0; i < NG * 2; ++i) {
        R.k[i] = R.valid ? kc[i] : make_uint4(0, 0, 0, 0);
        R.v[i] = R.valid ? vc[i] : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int G = 0; G < NG; ++G) {
        R.ks[G] = R.valid ? p.ks[row * NG + G] : 0;
        R.kb[G] = R.valid ? p.kb[row * NG + G] : 0;
        R.vs[G] = R.valid ? p.vs[row * NG + G] : 0;
        R.vb[G] = R.valid ? p.vb[row * NG + G] : 0;
      }
    };
    RawRow cur;
    if (n_tiles > 0) load_raw(0, cur);
    for (int j = 0; j < n_tiles; ++j) {
      const int buf = j & 1;         // TMEM S buffer
      const int kvb = j % LY::NKV;   // shared-memory K/V buffer, free once P . V(j - NKV) is done
      if (j >= LY::NKV && !*abort_flag) {
        if (!mbar_wait_bounded(bar(B_KVFREE + kvb), ((j - LY::NKV) / LY::NKV) & 1)) *abort_flag = 1;
      }
      // the producers decide together (no thread may be left waiting in barrier 1)
      if (group_bar_any(1, *abort_flag != 0)) break;
      RawRow nxt;
      if (j + 1 < n_tiles) load_raw(j + 1, nxt);
      uint8_t* kdst = smem + LY::OFF_K + kvb * LY::TILE;
      uint8_t* vdst = smem + LY::OFF_V + kvb * LY::TILE;
#pragma unroll
      for (int G = 0; G < NG; ++G) {
        const __half2 ks2 = scale_h2<SBF16>(cur.ks[G]), kb2 = scale_h2<SBF16>(cur.kb[G]);
        const __half2 vs2 = scale_h2<SBF16>(cur.vs[G]), vb2 = scale_h2<SBF16>(cur.vb[G]);
#pragma unroll
        for (int w4 = 0; w4 < 2; ++w4) {
          const uint4 kw = cur.k[G * 2 + w4], vw = cur.v[G * 2 + w4];
          const uint32_t kk[4] = {kw.x, kw.y, kw.z, kw.w};
          const uint32_t vv[4] = {vw.x, vw.y, vw.z, vw.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int wi = G * 8 + w4 * 4 + i;
            const uint32_t koff = (wi / 8) * (128 * 128) + r * 128 + (wi % 8) * 16;
            *reinterpret_cast<uint4*>(kdst + tc::swz(koff)) = dequant8(kk[i], ks2, kb2);
            const uint32_t voff = (wi / 8) * (128 * 128) + (r / 8) * 1024 + (r % 8) * 128 + (wi % 8) * 16;
            *reinterpret_cast<uint4*>(vdst + tc::swz(voff)) = dequant8(vv[i], vs2, vb2);
          }
        }
      }
      cur = nxt;
      tc::fence_proxy_async();
      named_bar_producers();
      if (r == 0) {
        tc::fence_after();
        bool ok = true;
        if (j >= 2) ok = mbar_wait_bounded(bar(B_SFREE + buf), ((j - 2) >> 1) & 1);
        if (ok) {
          const uint32_t kb_addr = sK + kvb * LY::TILE;
#pragma unroll
          for (int ks = 0; ks < KSTEPS; ++ks) {
            const uint32_t off = (ks / 4) * (128 * 128) + (ks % 4) * 32;
            tc::mma(tmem + buf * 128, tc::sdesc(sQ + off, 16, 1024), tc::sdesc(kb_addr + off, 16, 1024),
                    ID_S, ks > 0 ? 1u : 0u);
          }
          tc::commit(bar(B_SFULL + buf));
        } else {
          *abort_flag = 1;
        }
      }
    }
  } else {
    // ================================================================ softmax warps
    // Warp w owns S rows 32 (w % 4) .. +31 (its TMEM lane quarter) and key columns
    // 64 (w / 4) .. +63 of every tile; warps w and w + 4 share rows, exchange their row
    // maxima through shared memory (a 64-thread named barrier per pair) and keep partial
    // sums that are added at the end.  Each also rescales and writes back half of O.
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + (tid & 31);  // query row == TMEM lane
    const int lane_id = tid & 31;
    const int pair_bar = 3 + quarter;        // named barrier of warps quarter and quarter + 4
    const int rl = r / n_rep;
    const bool row_ok = r < tok_per_cta * n_rep && l0 + rl < p.q_len;
    const int l = l0 + (row_ok ? rl : 0);
    const int hq = h * n_rep + r % n_rep;
    const int pos = n - p.q_len + l;
    const int klo = max(st, p.window > 0 ? pos - p.window + 1 : 0);
    const int khi = p.causal ? min(n, pos + 1) : n;
    const int tlo = max(st, p.window > 0 ? pos_max - p.window + 1 : 0);  // CTA-wide safe range
    const int thi = p.causal ? min(n, pos_min + 1) : n;
    const float q_fac = sqf[r];
    const bool q_pos = q_fac >= 0.0f;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    float* rx = reinterpret_cast<float*>(smem + LY::OFF_RX);  // [2][128]
    constexpr int DH = D / 2;  // O columns this warp rescales and stores

    float m_run = -INFINITY, l_run = 0.0f;
    const uint32_t o_row = tmem + 256 + lane_base;  // this thread's row of the O accumulator
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

    // O accumulates in TMEM over all tiles (P . V with accumulate after the first tile);
    // a row's O is rescaled in TMEM only when its max moves by more than the slack.  Lane 0
    // of softmax warp 0 issues P . V of each tile once all rows of P are written (an
    // mbarrier of 256 arrivals), so the K/V buffer is released without waiting for the
    // producers' next dequantisation.  Every wait result is agreed by a warp pair through
    // an OR barrier, so both halves of a row leave together.
    for (int i = 0; i < n_tiles; ++i) {
      const int buf = i & 1;
      const int kvb = i % LY::NKV;
      const int t0 = lo + i * 128 + half * 64;  // first key of this warp's columns
      bool ok = !*abort_flag && mbar_wait_bounded(bar(B_SFULL + buf), (i >> 1) & 1);
      if (group_bar_any(pair_bar, !ok, 64)) {
        *abort_flag = 1;
        break;
      }
      tc::fence_after();
      const bool need_mask =
          __any_sync(0xffffffffu, DENSE || !row_ok || t0 < tlo || t0 + 64 > thi);  // warp-uniform
      float v[64];
      tc::tmem_ld64(tmem + buf * 128 + half * 64 + lane_base, v);
      if (need_mask) {
#pragma unroll
        for (int j2 = 0; j2 < 64; ++j2) v[j2] = masked(v[j2] * q_fac, t0 + j2);
      }
      float mp[8];
      const bool take_max = need_mask || q_pos;
#pragma unroll
      for (int k = 0; k < 8; ++k) mp[k] = take_max ? -INFINITY : INFINITY;
#pragma unroll
      for (int j2 = 0; j2 < 64; ++j2)
        mp[j2 & 7] = take_max ? fmaxf(mp[j2 & 7], v[j2]) : fminf(mp[j2 & 7], v[j2]);
#pragma unroll
      for (int k = 1; k < 8; ++k) mp[0] = take_max ? fmaxf(mp[0], mp[k]) : fminf(mp[0], mp[k]);
      const float my_max = need_mask ? mp[0] : mp[0] * q_fac;
      rx[half * 128 + r] = my_max;
      if (group_bar_any(pair_bar, false, 64)) {  // publishes rx between the pair
        *abort_flag = 1;
        break;
      }
      const float tile_max = fmaxf(my_max, rx[(half ^ 1) * 128 + r]);
      const bool raise = tile_max > m_run + kPrefillRescaleSlack;
      if (__any_sync(0xffffffffu, raise)) {  // the same rows, so the same answer in both halves
        const float m_new = raise ? tile_max : m_run;
        const float alpha = m_run == -INFINITY ? 0.0f : ex2(m_run - m_new);
        if (i >= 1) {
          // O is rescaled in TMEM only after P . V of the previous tile has landed in it
          if (__all_sync(0xffffffffu, mbar_wait_bounded(bar(B_OFULL), (i - 1) & 1))) {
            tc::fence_after();
            rescale_o<DH>(o_row + half * DH, alpha);
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
      // P (fp16 pairs) replaces this warp's own S columns: keys half * 64 + 2c, +1 in
      // column half * 64 + c of the tile's S buffer, the A operand of P . V
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float p0 = ex2(fmaf(v[2 * c], fac, -m_safe));
        const float p1 = ex2(fmaf(v[2 * c + 1], fac, -m_safe));
        lp[(2 * c) & 7] += p0;
        lp[(2 * c + 1) & 7] += p1;
        pk[c] = pack_half2(p0, p1);
      }
      tc::tmem_st32u(tmem + buf * 128 + half * 64 + lane_base, pk);
#pragma unroll
      for (int k = 0; k < 8; ++k) l_run += lp[k];
      tc::fence_before();
      mbar_arrive(bar(B_PFULL));
      if (warp == 0) {
        // a failed wait only raises the flag: warp 0 must not leave its pair (warp 4)
        // waiting in their barrier, so both see the flag at the next pair barrier
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar(B_PFULL), i & 1));
        if (!ok) *abort_flag = 1;
        if (ok && !*abort_flag && lane_id == 0) {
          tc::fence_after();
          const uint32_t vb_addr = sV + kvb * LY::TILE;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            // 16 keys per step: columns (ks / 4) * 64 + (ks % 4) * 8 of the S buffer
            tc::mma_ts(tmem + 256, tmem + buf * 128 + (ks / 4) * 64 + (ks % 4) * 8,
                       tc::sdesc(vb_addr + ks * 2048, 128 * 128, 1024), ID_O, (i > 0 || ks > 0) ? 1u : 0u);
          }
          tc::commit(bar(B_OFULL));
          tc::commit(bar(B_KVFREE + kvb));
          tc::commit(bar(B_SFREE + buf));
        }
        __syncwarp();
      }
    }
    // ---- epilogue: this thread's half of its output row.  The pair adds its partial sums
    // (the OR barrier also publishes them); O columns arrive in perm8 order within each
    // 8-dim chunk and are put back before the store.
    bool fin = n_tiles > 0 && !*abort_flag;
    if (fin) fin = mbar_wait_bounded(bar(B_OFULL), (n_tiles - 1) & 1);
    fin = __all_sync(0xffffffffu, fin);
    rx[half * 128 + r] = l_run;
    const bool bad = group_bar_any(pair_bar, !fin, 64);
    if (!bad) {
      tc::fence_after();
      float o_acc[DH];
#pragma unroll
      for (int c = 0; c < DH / 32; ++c) {
        float t32[32];
        tc::tmem_ld32(o_row + half * DH + c * 32, t32);
#pragma unroll
        for (int j2 = 0; j2 < 32; ++j2) o_acc[c * 32 + j2] = t32[j2];
      }
      if (row_ok) {
        const float l_tot = rx[r] + rx[128 + r];
#pragma unroll
        for (int c8 = 0; c8 < DH / 8; ++c8) {
          float t8[8];
#pragma unroll
          for (int q8 = 0; q8 < 8; ++q8) t8[q8] = o_acc[c8 * 8 + q8];
#pragma unroll
          for (int q8 = 0; q8 < 8; ++q8) o_acc[c8 * 8 + perm8(q8)] = t8[q8];
        }
        const bool sink = p.sinks != nullptr;
        const float inv =
            softmax_out_factor(m_run, l_tot, sink, sink ? p.sinks[hq] * 1.4426950408889634f : 0.0f);
        const int64_t ob = (int64_t)b * p.osb + (int64_t)hq * p.osh + (int64_t)l * p.osl + half * DH;
        if (p.out_dtype == AM_DTYPE_F32) {
          float* o = static_cast<float*>(p.out) + ob;
          if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
            for (int d = 0; d < DH; d += 4)
              *reinterpret_cast<float4*>(o + d) =
                  make_float4(o_acc[d] * inv, o_acc[d + 1] * inv, o_acc[d + 2] * inv, o_acc[d + 3] * inv);
          } else {
#pragma unroll
            for (int d = 0; d < DH; ++d) o[d] = o_acc[d] * inv;
          }
        } else {
          const bool bf = p.out_dtype == AM_DTYPE_BF16;
          uint16_t* o = static_cast<uint16_t*>(p.out) + ob;
          if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
            for (int d = 0; d < DH; d += 8) {
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
            for (int d = 0; d < DH; ++d) o[d] = bf ? f2h<true>(o_acc[d] * inv) : f2h<false>(o_acc[d] * inv);
          }
        }
      }
    } else {
      *abort_flag = 1;
    }
  }

  if (*abort_flag && tid == 0) flag_status(p.status, AM_STATUS_TIMEOUT);
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                 "r"(LY::TMEM_COLS));
  }
}

bool prefill_supported(int k_dim, int v_dim) {
  return k_dim == v_dim && (k_dim == 64 || k_dim == 128);
}

template <int D, bool SBF16, bool PAGED, bool DENSE>
static cudaError_t launch_prefill_t(const DecodeParams& p, int batch, cudaStream_t stream) {
  using LY = PrefillLayout<D>;
  auto kfn = prefill_kernel<D, SBF16, PAGED, DENSE>;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, LY::SMEM);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  const int tok_per_cta = 128 / p.n_rep;
  dim3 grid(p.hkv, batch, (p.q_len + tok_per_cta - 1) / tok_per_cta);
  kfn<<<grid, kPrefillThreads, LY::SMEM, stream>>>(p);
  return cudaGetLastError();
}

template <int D, bool SBF16, bool PAGED>
static cudaError_t launch_prefill_m(const DecodeParams& p, int batch, cudaStream_t stream) {
  return p.mask_kind != AM_MASK_NONE ? launch_prefill_t<D, SBF16, PAGED, true>(p, batch, stream)
                                     : launch_prefill_t<D, SBF16, PAGED, false>(p, batch, stream);
}

cudaError_t launch_prefill(const DecodeParams& p, int batch, bool paged, bool scale_bf16,
                           cudaStream_t stream) {
  if (p.n_rep < 1 || p.n_rep > 128) return cudaErrorNotSupported;
  if (p.k_dim == 128 && p.v_dim == 128) {
    if (paged) return scale_bf16 ? launch_prefill_m<128, true, true>(p, batch, stream)
                                 : launch_prefill_m<128, false, true>(p, batch, stream);
    return scale_bf16 ? launch_prefill_m<128, true, false>(p, batch, stream)
                      : launch_prefill_m<128, false, false>(p, batch, stream);
  }
  if (p.k_dim == 64 && p.v_dim == 64) {
    if (paged) return scale_bf16 ? launch_prefill_m<64, true, true>(p, batch, stream)
                                 : launch_prefill_m<64, false, true>(p, batch, stream);
    return scale_bf16 ? launch_prefill_m<64, true, false>(p, batch, stream)
                      : launch_prefill_m<64, false, false>(p, batch, stream);
  }
  return cudaErrorNotSupported;
}

}  // namespace am
