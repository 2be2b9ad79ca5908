// Affine 4-bit quantization (group 64) on the GPU: plain quantize, dequantize, and the
// fused quantize-on-append that scatters into a contiguous or paged Q4 cache.
//
// Quantization rule (mlx 0.30.3 affine quantizer, restated; the reference calls it at
// src/agent_memory/adapters/outbound/mlx_quantized_extensions.py:273-274), per 64-element
// group in fp32 with IEEE-rounded division:
//   scale = max((max - min) / 15, 1e-7); the endpoint with the larger magnitude is the
//   "edge" (scale negated when the edge is the max); q0 = rint(edge / scale); when q0 != 0
//   the scale becomes edge / q0 and the bias the edge (zero is then exactly representable),
//   otherwise bias = 0; code = clamp(rint((w - bias) / scale), 0, 15).
// Scale and bias are stored in the input dtype; codes are packed 8 per uint32, LSB first.
//
// Work mapping: 8 lanes own one 64-element group (16-byte load each, one output word
// each); a warp covers 4 groups.  Min/max are reduced with 3 xor-shuffles inside the
// 8-lane team.  The kernels are HBM-bound: 128 B read + 36 B written per group (fp16).
#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "am_common.cuh"
#include "am_internal.h"

namespace am {

template <bool BF16>
__device__ __forceinline__ void load8(const uint16_t* src, float (&w)[8]) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(src));
  const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    w[2 * i] = h2f<BF16>(static_cast<uint16_t>(u[i] & 0xffffu));
    w[2 * i + 1] = h2f<BF16>(static_cast<uint16_t>(u[i] >> 16));
  }
}

// Quantize the 64-element group spread over the 8 lanes of a team (8 values per lane).
// Every lane of the warp must call this (shuffles use the full mask).
__device__ __forceinline__ uint32_t quantize_team(const float (&w)[8], float& scale_out,
                                                  float& bias_out) {
  float mn = w[0], mx = w[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    mn = fminf(mn, w[i]);
    mx = fmaxf(mx, w[i]);
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const bool side = fabsf(mn) > fabsf(mx);
  float scale = fmaxf(__fdiv_rn(__fsub_rn(mx, mn), 15.0f), 1e-7f);
  scale = side ? scale : -scale;
  const float edge = side ? mn : mx;
  // q0 = rint(fl(edge / scale)); |edge / scale| <= 15, so the reciprocal product decides it
  // except within 2^-16 of a half-integer (see the codes below)
  float q0;
  {
    const float t = __fmul_rn(edge, __frcp_rn(scale));
    q0 = rintf(t);
    if (fabsf(t - q0) > 0.5f - 1.52587890625e-05f) q0 = rintf(__fdiv_rn(edge, scale));
  }
  float bias = 0.0f;
  if (q0 != 0.0f) {
    scale = __fdiv_rn(edge, q0);
    bias = edge;
  }
  // code = clamp(rint(fl((w - bias) / scale)), 0, 15) with the IEEE-rounded quotient.  The
  // product with the correctly rounded reciprocal is within 2^-19 of the exact quotient for
  // |quotient| < 16 (two roundings of 2^-24 relative each), so its rint can only differ from
  // the rint of the rounded quotient within that distance of a half-integer: there (and only
  // there) the division itself is done.  Quotients of 16 and more clamp to 15 either way.
  // The rounding itself stays on the FMA/ALU pipes: t is first clamped to [-1, 16] (codes of
  // quotients below -0.5 are 0 and above 15.5 are 15 either way; NaN clamps to -1 -> 0, as
  // fmaxf(rint(NaN), 0) does), then adding 1.5 * 2^23 rounds it to the nearest integer (ties
  // to even, as rint) in the low mantissa bits.
  const float inv = __frcp_rn(scale);
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float d = __fsub_rn(w[i], bias);
    float t = fminf(fmaxf(__fmul_rn(d, inv), -1.0f), 16.0f);
    const float big = __fadd_rn(t, 12582912.0f);
    if (fabsf(t - __fsub_rn(big, 12582912.0f)) > 0.5f - 1.52587890625e-05f) {  // 0.5 - 2^-16
      t = fminf(fmaxf(__fdiv_rn(d, scale), -1.0f), 16.0f);
      const int c = __float_as_int(__fadd_rn(t, 12582912.0f)) - 0x4B400000;
      packed |= static_cast<uint32_t>(min(max(c, 0), 15)) << (4 * i);
    } else {
      const int c = __float_as_int(big) - 0x4B400000;
      packed |= static_cast<uint32_t>(min(max(c, 0), 15)) << (4 * i);
    }
  }
  scale_out = scale;
  bias_out = bias;
  return packed;
}

template <bool BF16>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const uint16_t* __restrict__ x,
                                                            int64_t n_groups, int dim,
                                                            uint32_t* __restrict__ codes,
                                                            uint16_t* __restrict__ scales,
                                                            uint16_t* __restrict__ biases) {
  const int lane = threadIdx.x & 31;
  const int team = lane >> 3, sub = lane & 7;
  const int64_t warps_total = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t warp0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  for (int64_t wg = warp0; wg * 4 < n_groups; wg += warps_total) {
    const int64_t gi = wg * 4 + team;
    const bool active = gi < n_groups;
    float w[8];
    if (active) {
      load8<BF16>(x + gi * kGroup + sub * 8, w);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) w[i] = 0.0f;
    }
    float s, b;
    const uint32_t packed = quantize_team(w, s, b);
    if (active) {
      codes[gi * 8 + sub] = packed;
      if (sub == 0) {
        scales[gi] = f2h<BF16>(s);
        biases[gi] = f2h<BF16>(b);
      }
    }
  }
  (void)dim;
}

template <bool BF16>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint32_t* __restrict__ codes,
                                                         const uint16_t* __restrict__ scales,
                                                         const uint16_t* __restrict__ biases,
                                                         int64_t n_words, void* __restrict__ out,
                                                         int out_dtype) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_words;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t word = codes[i];
    const int64_t grp = i >> 3;
    const float s = h2f<BF16>(scales[grp]);
    const float b = h2f<BF16>(biases[grp]);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      store_out(out, i * 8 + k, fmaf(static_cast<float>((word >> (4 * k)) & 0xfu), s, b),
                out_dtype);
    }
  }
}

// Quantize-on-append.  An 8-lane team owns one new row (b, h, l): it loads every K and V
// group of the row (16 bytes per lane per group, all loads issued before any arithmetic),
// resolves the destination row once, then quantizes and stores group by group.  A warp
// covers 4 rows; index arithmetic is 32-bit (the launcher refuses more than 2^31 rows).
constexpr int kMaxGroupsPerRow = 4;  // head dims up to 256

template <bool BF16>
__global__ void __launch_bounds__(256) append_kernel(AppendParams p) {
  const int lane = threadIdx.x & 31;
  const int team = lane >> 3, sub = lane & 7;
  const int ngk = p.k_dim / kGroup, ngv = p.v_dim / kGroup;
  const int rows = p.batch * p.hkv * p.n_new;
  const int warps_total = gridDim.x * (blockDim.x >> 5);
  const int warp0 = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  for (int wr = warp0; wr < (rows + 3) / 4; wr += warps_total) {
    const int row = wr * 4 + team;
    const bool active = row < rows;
    const int bh = active ? row / p.n_new : 0;
    const int l = active ? row - bh * p.n_new : 0;
    const int b = bh / p.hkv;
    const int h = bh - b * p.hkv;
    uint4 rk[kMaxGroupsPerRow], rv[kMaxGroupsPerRow];
    {
      const uint16_t* ksrc = p.k + b * p.ksb + h * p.ksh + l * p.ksl + sub * 8;
      const uint16_t* vsrc = p.v + b * p.vsb + h * p.vsh + l * p.vsl + sub * 8;
#pragma unroll
      for (int g = 0; g < kMaxGroupsPerRow; ++g) {
        rk[g] = (active && g < ngk) ? __ldg(reinterpret_cast<const uint4*>(ksrc + g * kGroup)) : make_uint4(0, 0, 0, 0);
        rv[g] = (active && g < ngv) ? __ldg(reinterpret_cast<const uint4*>(vsrc + g * kGroup)) : make_uint4(0, 0, 0, 0);
      }
    }
    // destination row (-1: skipped and flagged)
    int64_t drow = -1;
    if (active) {
      const int64_t pos = (int64_t)p.positions[b] + l;
      if (p.layout == AM_LAYOUT_PAGED) {
        if (pos < 0 || pos / p.block_tokens >= p.table_stride) {
          if (sub == 0) flag_status(p.status, AM_STATUS_BAD_POSITION);
        } else {
          const int pi = static_cast<int>(pos);
          const int bi = pi / p.block_tokens;
          const int32_t blk = p.table[(int64_t)b * p.table_stride + bi];
          if (blk < 0 || blk >= p.capacity) {
            if (sub == 0) flag_status(p.status, AM_STATUS_BAD_BLOCK);
          } else {
            drow = ((int64_t)blk * p.hkv + h) * p.block_tokens + (pi - bi * p.block_tokens);
          }
        }
      } else if (pos < 0 || pos >= p.capacity) {
        if (sub == 0) flag_status(p.status, AM_STATUS_BAD_POSITION);
      } else {
        drow = ((int64_t)b * p.hkv + h) * p.capacity + pos;
      }
    }
    // every lane of the warp runs every quantize_team (its shuffles use the full mask); the
    // group counts are the same for all rows
#pragma unroll
    for (int g = 0; g < 2 * kMaxGroupsPerRow; ++g) {
      const bool is_v = g >= kMaxGroupsPerRow;
      const int gg = is_v ? g - kMaxGroupsPerRow : g;
      const int ng = is_v ? ngv : ngk;
      if (gg >= ng) continue;  // uniform across the warp
      const uint4 raw = is_v ? rv[gg] : rk[gg];
      const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
      float w[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        w[2 * i] = h2f<BF16>(static_cast<uint16_t>(u[i] & 0xffffu));
        w[2 * i + 1] = h2f<BF16>(static_cast<uint16_t>(u[i] >> 16));
      }
      float sc, bias;
      const uint32_t packed = quantize_team(w, sc, bias);
      if (drow < 0) continue;
      uint32_t* codes = is_v ? p.vc : p.kc;
      uint16_t* scales = is_v ? p.vs : p.ks;
      uint16_t* biases = is_v ? p.vb : p.kb;
      codes[drow * (ng * 8) + gg * 8 + sub] = packed;
      if (sub == 0) {
        scales[drow * ng + gg] = f2h<BF16>(sc);
        biases[drow * ng + gg] = f2h<BF16>(bias);
      }
    }
  }
}

static int grid_for(int64_t warps_needed, int warps_per_block) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    sms = 148;
    (void)cudaGetLastError();  // clear: this query must not poison a later launch check
  }
  const int64_t blocks = (warps_needed + warps_per_block - 1) / warps_per_block;
  const int64_t cap = (int64_t)sms * 16;  // grid-stride beyond 16 blocks of 256 per SM
  return static_cast<int>(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

cudaError_t launch_quantize(const void* x, bool bf16, int64_t rows, int dim, uint32_t* codes,
                            void* scales, void* biases, cudaStream_t stream) {
  const int64_t n_groups = rows * (dim / kGroup);
  if (n_groups == 0) return cudaSuccess;
  const int grid = grid_for((n_groups + 3) / 4, 8);
  if (bf16) {
    quantize_rows_kernel<true><<<grid, 256, 0, stream>>>(
        static_cast<const uint16_t*>(x), n_groups, dim, codes, static_cast<uint16_t*>(scales),
        static_cast<uint16_t*>(biases));
  } else {
    quantize_rows_kernel<false><<<grid, 256, 0, stream>>>(
        static_cast<const uint16_t*>(x), n_groups, dim, codes, static_cast<uint16_t*>(scales),
        static_cast<uint16_t*>(biases));
  }
  return cudaGetLastError();
}

cudaError_t launch_dequantize(const uint32_t* codes, const void* scales, const void* biases,
                              bool bf16, int64_t rows, int dim, void* out, int out_dtype,
                              cudaStream_t stream) {
  const int64_t n_words = rows * (dim / 8);
  if (n_words == 0) return cudaSuccess;
  const int grid = grid_for((n_words + 31) / 32, 8);
  if (bf16) {
    dequantize_kernel<true><<<grid, 256, 0, stream>>>(
        codes, static_cast<const uint16_t*>(scales), static_cast<const uint16_t*>(biases),
        n_words, out, out_dtype);
  } else {
    dequantize_kernel<false><<<grid, 256, 0, stream>>>(
        codes, static_cast<const uint16_t*>(scales), static_cast<const uint16_t*>(biases),
        n_words, out, out_dtype);
  }
  return cudaGetLastError();
}

cudaError_t launch_append(const AppendParams& p, bool bf16, cudaStream_t stream) {
  const int64_t rows = (int64_t)p.batch * p.hkv * p.n_new;
  const int64_t n_groups = rows * (p.k_dim / kGroup + p.v_dim / kGroup);
  if (n_groups == 0) return cudaSuccess;
  if (rows + 3 > INT32_MAX || p.k_dim > kMaxGroupsPerRow * kGroup || p.v_dim > kMaxGroupsPerRow * kGroup)
    return cudaErrorNotSupported;  // 32-bit row indices; head dims up to 256
  const int grid = grid_for((rows + 3) / 4, 8);
  if (bf16) {
    append_kernel<true><<<grid, 256, 0, stream>>>(p);
  } else {
    append_kernel<false><<<grid, 256, 0, stream>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace am
