// Chunked-prefill attention over a Q4 cache on 5th-generation tensor cores (tcgen05).
//
// One CTA = 128 query rows of one KV head of one sequence.  Rows are (token, GQA head)
// pairs, token-major: 128 / n_rep query tokens times the n_rep heads that share the KV
// head, so each dequantized K/V tile feeds all of them.  Per 128-token KV tile:
//   1. the 128 threads dequantize the Q4 K and V rows (one token each) into fp16
//      operand tiles in shared memory (128-byte swizzle; K K-major, V MN-major);
//   2. one thread issues S = Q . K^T as D/16 tcgen05.mma (M=128, N=128, K=16, fp32
//      accumulators in TMEM columns [0,128)) and commits to an mbarrier;
//   3. thread r reads TMEM lane r (its row of S) with tcgen05.ld, applies scale and mask,
//      updates the running max / sum and writes P (fp16) into the K tile's buffer;
//   4. one thread issues O_tile = P . V (8 MMAs, TMEM columns [128, 128+D)); each thread
//      then adds its TMEM row of O_tile to its fp32 register accumulator.
// Operands are fp16 for every query dtype: bf16 queries are rescaled per row by a power
// of two so the conversion is exact, and the factor is removed from S in fp32.
// Every mbarrier wait is bounded (2 s of %globaltimer); on timeout the kernel flags
// AM_STATUS_TIMEOUT, stops issuing work, frees its TMEM and returns.
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

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if (globaltimer() - t0 > 2000000000ull) return false;
  }
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

// Byte offset inside a 1024-byte-aligned 128B-swizzled region.
__device__ __forceinline__ uint32_t swz(uint32_t off) { return off ^ (((off >> 7) & 7u) << 4); }

}  // namespace tc

template <int D>
struct PrefillLayout {
  static constexpr int TILE_BYTES = 128 * D * 2;                       // 128 rows x D fp16
  static constexpr int P_BYTES = 128 * 128 * 2;                        // 128 rows x 128 keys
  static constexpr int KP_BYTES = TILE_BYTES > P_BYTES ? TILE_BYTES : P_BYTES;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + TILE_BYTES;  // K tile, reused for P
  static constexpr int OFF_V = OFF_K + KP_BYTES;
  static constexpr int OFF_BAR = OFF_V + TILE_BYTES;
  static constexpr int SMEM = OFF_BAR + 64 + 1024;  // + slack for 1024-byte alignment
  static constexpr uint32_t TMEM_COLS = 256;
};

__device__ __forceinline__ uint32_t pack_h2(float a, float b) { return pack_half2(a, b); }

template <int D, bool SBF16, bool PAGED>
__global__ void __launch_bounds__(128) prefill_kernel(const DecodeParams p) {
  using LY = PrefillLayout<D>;
  constexpr int NG = D / 64;
  constexpr int KSTEPS = D / 16;

  extern __shared__ uint8_t smem_raw[];
  // 1024-byte-align the operand region (swizzle atoms).
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_addr & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  const uint32_t s_base = raw_addr + pad;
  const uint32_t sQ = s_base + LY::OFF_Q, sK = s_base + LY::OFF_K, sV = s_base + LY::OFF_V;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + LY::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + LY::OFF_BAR + 8);
  int* abort_flag = reinterpret_cast<int*>(smem + LY::OFF_BAR + 16);
  const uint32_t bar_addr = smem_u32(bar);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int b = blockIdx.z, h = blockIdx.y;
  const int n_rep = p.n_rep;
  const int tok_per_cta = 128 / n_rep;
  const int l0 = blockIdx.x * tok_per_cta;
  const int l_last = min(l0 + tok_per_cta, p.q_len) - 1;

  const int n = p.kv_len[b];
  const int st = p.kv_start != nullptr ? p.kv_start[b] : 0;
  const bool dense_mask = p.mask_kind != AM_MASK_NONE;
  const int pos_min = n - p.q_len + l0, pos_max = n - p.q_len + l_last;
  int lo = 0, hi = n;
  if (!dense_mask) {
    lo = max(st, 0);
    if (p.window > 0) lo = max(lo, pos_min - p.window + 1);
  }
  if (p.causal) hi = min(hi, pos_max + 1);

  // ---- this thread's query row
  const int r = tid;
  const int rl = r / n_rep;
  const bool row_ok = r < tok_per_cta * n_rep && l0 + rl < p.q_len;
  const int l = l0 + (row_ok ? rl : 0);
  const int hq = h * n_rep + r % n_rep;
  const int pos = n - p.q_len + l;

  // ---- setup: barrier, TMEM, Q tile
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar_addr), "r"(1));
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    *abort_flag = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(LY::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  // Q row -> fp16 with a power-of-two prescale (exact for fp16 and bf16 inputs).
  float q_fac;
  {
    const uint16_t* qrow = p.q + (int64_t)b * p.qsb + (int64_t)hq * p.qsh + (int64_t)l * p.qsl;
    float amax = 0.0f;
    if (row_ok) {
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
    q_fac = p.scale_log2 / pw;
    for (int c = 0; c < D / 8; ++c) {
      uint4 outv = make_uint4(0, 0, 0, 0);
      if (row_ok) {
        const uint4 raw = *reinterpret_cast<const uint4*>(qrow + c * 8);
        const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
        uint32_t o4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          o4[i] = pack_h2(h2f_rt(u[i] & 0xffffu, p.q_bf16) * pw, h2f_rt(u[i] >> 16, p.q_bf16) * pw);
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
  const uint32_t tmem_s = tmem;        // S: columns [0, 128)
  const uint32_t tmem_o = tmem + 128;  // O tile: columns [128, 128 + D)
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;

  float o_acc[D];
#pragma unroll
  for (int i = 0; i < D; ++i) o_acc[i] = 0.0f;
  float m_run = -INFINITY, l_run = 0.0f;
  uint32_t phase = 0;
  bool aborted = false;

  constexpr uint32_t ID_S = tc::idesc(128, 128, false);
  constexpr uint32_t ID_O = tc::idesc(128, D, true);

  for (int t0 = lo; t0 < hi && !aborted; t0 += 128) {
    // ---- 1. dequantize K and V rows (token t0 + tid)
    {
      const int tok = t0 + tid;
      bool valid = tok < n && tok >= 0;
      int64_t row = 0;
      if (valid) {
        if constexpr (PAGED) {
          const int bi = tok / p.block_tokens;
          const int32_t blk = bi < p.table_stride ? p.table[(int64_t)b * p.table_stride + bi] : -1;
          if (blk < 0 || blk >= p.capacity) {
            valid = false;
            flag_status(p.status, AM_STATUS_BAD_BLOCK);
          } else {
            row = ((int64_t)blk * p.hkv + h) * p.block_tokens + tok % p.block_tokens;
          }
        } else {
          row = ((int64_t)b * p.hkv + h) * p.capacity + tok;
        }
      }
      const uint32_t* kc = p.kc + row * (D / 8);
      const uint32_t* vc = p.vc + row * (D / 8);
#pragma unroll
      for (int G = 0; G < NG; ++G) {
        float ks = 0.f, kb = 0.f, vs = 0.f, vb = 0.f;
        if (valid) {
          ks = h2f<SBF16>(p.ks[row * NG + G]);
          kb = h2f<SBF16>(p.kb[row * NG + G]);
          vs = h2f<SBF16>(p.vs[row * NG + G]);
          vb = h2f<SBF16>(p.vb[row * NG + G]);
        }
#pragma unroll
        for (int w4 = 0; w4 < 2; ++w4) {  // 8 words per group, loaded 4 at a time
          uint4 kw = make_uint4(0, 0, 0, 0), vw = make_uint4(0, 0, 0, 0);
          if (valid) {
            kw = *reinterpret_cast<const uint4*>(kc + G * 8 + w4 * 4);
            vw = *reinterpret_cast<const uint4*>(vc + G * 8 + w4 * 4);
          }
          const uint32_t kk[4] = {kw.x, kw.y, kw.z, kw.w};
          const uint32_t vv[4] = {vw.x, vw.y, vw.z, vw.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int wi = G * 8 + w4 * 4 + i;  // word index = 8-element chunk along D
            uint32_t ko[4], vo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float k0 = valid ? fmaf(static_cast<float>((kk[i] >> (8 * e)) & 0xfu), ks, kb) : 0.f;
              const float k1 = valid ? fmaf(static_cast<float>((kk[i] >> (8 * e + 4)) & 0xfu), ks, kb) : 0.f;
              const float v0 = valid ? fmaf(static_cast<float>((vv[i] >> (8 * e)) & 0xfu), vs, vb) : 0.f;
              const float v1 = valid ? fmaf(static_cast<float>((vv[i] >> (8 * e + 4)) & 0xfu), vs, vb) : 0.f;
              ko[e] = pack_h2(k0, k1);
              vo[e] = pack_h2(v0, v1);
            }
            // K: K-major [token][dim], 64-dim column blocks of 128 rows x 128 B.
            const uint32_t koff = (wi / 8) * (128 * 128) + tid * 128 + (wi % 8) * 16;
            *reinterpret_cast<uint4*>(smem + LY::OFF_K + tc::swz(koff)) =
                make_uint4(ko[0], ko[1], ko[2], ko[3]);
            // V: MN-major [token][dim]: 64-dim blocks (LBO = 16 KB) of 8-token atoms (SBO = 1 KB).
            const uint32_t voff = (wi / 8) * (128 * 128) + (tid / 8) * 1024 + (tid % 8) * 128 + (wi % 8) * 16;
            *reinterpret_cast<uint4*>(smem + LY::OFF_V + tc::swz(voff)) =
                make_uint4(vo[0], vo[1], vo[2], vo[3]);
          }
        }
      }
    }
    tc::fence_proxy_async();
    tc::fence_before();
    __syncthreads();
    // ---- 2. S = Q . K^T
    if (tid == 0) {
      tc::fence_after();
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks) {
        const uint32_t koff = (ks / 4) * (128 * 128) + (ks % 4) * 32;
        tc::mma(tmem_s, tc::sdesc(sQ + koff, 16, 1024), tc::sdesc(sK + koff, 16, 1024), ID_S,
                ks > 0 ? 1u : 0u);
      }
      tc::commit(bar_addr);
    }
    bool ok = tc::mbar_wait(bar_addr, phase);
    phase ^= 1u;
    if (!__syncthreads_and(ok)) {
      aborted = true;
      break;
    }
    tc::fence_after();

    // ---- 3. softmax on this thread's row of S
    const bool need_mask = dense_mask || t0 < st || t0 + 127 >= n ||
                           (p.causal && t0 + 127 > pos_min) ||
                           (p.window > 0 && t0 <= pos_max - p.window);
    auto masked_val = [&](float s, int j) -> float {
      const int tok = t0 + j;
      bool keep = row_ok && tok < n && tok >= st;
      if (p.causal && tok > pos) keep = false;
      if (p.window > 0 && tok <= pos - p.window) keep = false;
      if (!keep) return -INFINITY;
      if (dense_mask) {
        const int64_t idx = (int64_t)b * p.msb + (int64_t)hq * p.msh + (int64_t)l * p.msl +
                            (int64_t)tok * p.msn;
        if (p.mask_kind == AM_MASK_BOOL) {
          if (static_cast<const uint8_t*>(p.mask)[idx] == 0) return -1.0e30f;
        } else {
          float mv = p.mask_dtype == AM_DTYPE_F32
                         ? static_cast<const float*>(p.mask)[idx]
                         : h2f_rt(static_cast<const uint16_t*>(p.mask)[idx],
                                  p.mask_dtype == AM_DTYPE_BF16);
          s = fmaf(mv, 1.4426950408889634f, s);
        }
      }
      return s;
    };
    float tile_max = -INFINITY;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float v[32];
      tc::tmem_ld32(tmem_s + lane_base + c * 32, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float s = v[j] * q_fac;
        if (need_mask) s = masked_val(s, c * 32 + j);
        tile_max = fmaxf(tile_max, s);
      }
    }
    const float m_new = fmaxf(m_run, tile_max);
    if (m_new > m_run) {
      const float alpha = m_run == -INFINITY ? 0.0f : ex2(m_run - m_new);
#pragma unroll
      for (int i = 0; i < D; ++i) o_acc[i] *= alpha;
      l_run *= alpha;
      m_run = m_new;
    }
    const float m_safe = m_run == -INFINITY ? 0.0f : m_run;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float v[32];
      tc::tmem_ld32(tmem_s + lane_base + c * 32, v);
      uint32_t pk[16];
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        float s0 = v[j] * q_fac, s1 = v[j + 1] * q_fac;
        if (need_mask) {
          s0 = masked_val(s0, c * 32 + j);
          s1 = masked_val(s1, c * 32 + j + 1);
        }
        const float p0 = ex2(s0 - m_safe), p1 = ex2(s1 - m_safe);
        l_run += p0 + p1;
        pk[j / 2] = pack_h2(p0, p1);
      }
      // P row r, keys c*32 .. c*32+31: K-major over keys, 64-key column blocks.
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const int key0 = c * 32 + q4 * 8;
        const uint32_t off = (key0 / 64) * (128 * 128) + r * 128 + ((key0 % 64) / 8) * 16;
        *reinterpret_cast<uint4*>(smem + LY::OFF_K + tc::swz(off)) =
            make_uint4(pk[q4 * 4], pk[q4 * 4 + 1], pk[q4 * 4 + 2], pk[q4 * 4 + 3]);
      }
    }
    tc::fence_proxy_async();
    tc::fence_before();
    __syncthreads();
    // ---- 4. O_tile = P . V
    if (tid == 0) {
      tc::fence_after();
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t poff = (ks / 4) * (128 * 128) + (ks % 4) * 32;
        tc::mma(tmem_o, tc::sdesc(sK + poff, 16, 1024), tc::sdesc(sV + ks * 2048, 128 * 128, 1024),
                ID_O, ks > 0 ? 1u : 0u);
      }
      tc::commit(bar_addr);
    }
    ok = tc::mbar_wait(bar_addr, phase);
    phase ^= 1u;
    if (!__syncthreads_and(ok)) {
      aborted = true;
      break;
    }
    tc::fence_after();
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      float v[32];
      tc::tmem_ld32(tmem_o + lane_base + c * 32, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) o_acc[c * 32 + j] += v[j];
    }
    tc::fence_before();
    __syncthreads();  // TMEM S / O and the K, V, P buffers are free for the next tile
  }

  if (aborted) {
    if (tid == 0) flag_status(p.status, AM_STATUS_TIMEOUT);
    // Give in-flight MMAs a bounded chance to drain before the TMEM is released.
    tc::mbar_wait(bar_addr, phase);
  }

  // ---- epilogue
  if (row_ok && !aborted) {
    const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
    const int64_t ob = (int64_t)b * p.osb + (int64_t)hq * p.osh + (int64_t)l * p.osl;
#pragma unroll
    for (int d = 0; d < D; ++d) store_out(p.out, ob + d, o_acc[d] * inv, p.out_dtype);
  }
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

template <int D, bool SBF16, bool PAGED>
static cudaError_t launch_prefill_t(const DecodeParams& p, int batch, cudaStream_t stream) {
  using LY = PrefillLayout<D>;
  auto kfn = prefill_kernel<D, SBF16, PAGED>;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, LY::SMEM);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  const int tok_per_cta = 128 / p.n_rep;
  dim3 grid((p.q_len + tok_per_cta - 1) / tok_per_cta, p.hkv, batch);
  kfn<<<grid, 128, LY::SMEM, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_prefill(const DecodeParams& p, int batch, bool paged, bool scale_bf16,
                           cudaStream_t stream) {
  if (p.n_rep < 1 || p.n_rep > 128) return cudaErrorNotSupported;
  if (p.k_dim == 128 && p.v_dim == 128) {
    if (paged) return scale_bf16 ? launch_prefill_t<128, true, true>(p, batch, stream)
                                 : launch_prefill_t<128, false, true>(p, batch, stream);
    return scale_bf16 ? launch_prefill_t<128, true, false>(p, batch, stream)
                      : launch_prefill_t<128, false, false>(p, batch, stream);
  }
  if (p.k_dim == 64 && p.v_dim == 64) {
    if (paged) return scale_bf16 ? launch_prefill_t<64, true, true>(p, batch, stream)
                                 : launch_prefill_t<64, false, true>(p, batch, stream);
    return scale_bf16 ? launch_prefill_t<64, true, false>(p, batch, stream)
                      : launch_prefill_t<64, false, false>(p, batch, stream);
  }
  return cudaErrorNotSupported;
}

}  // namespace am
