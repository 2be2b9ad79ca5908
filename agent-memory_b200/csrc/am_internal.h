// Internal launcher declarations shared by the kernel files and the C-ABI layer.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "am_q4.h"

namespace am {

struct AppendParams;
struct DecodeParams;
struct BlockCopyParams;
struct BlockListParams;

cudaError_t launch_quantize(const void* x, bool bf16, int64_t rows, int dim, uint32_t* codes,
                            void* scales, void* biases, cudaStream_t stream);
cudaError_t launch_dequantize(const uint32_t* codes, const void* scales, const void* biases,
                              bool bf16, int64_t rows, int dim, void* out, int out_dtype,
                              cudaStream_t stream);
cudaError_t launch_append(const AppendParams& p, bool bf16, cudaStream_t stream);

// Decode: returns cudaErrorNotSupported (without launching) for head dims without a kernel.
bool decode_supported(int k_dim, int v_dim);
// Tokens per decode pipeline stage for a head-dim pair (paged blocks must hold a whole stage).
int decode_stage_tokens(int k_dim, int v_dim);
cudaError_t launch_decode(const DecodeParams& p, int batch, int row_groups, bool paged,
                          bool scale_bf16, cudaStream_t stream);

bool prefill_supported(int k_dim, int v_dim);
// Keys per tile of the prefill attention kernel for a head-dim pair (the tensor-map box rows).
int prefill_key_tile(int k_dim, int v_dim);
// True when the attention kernel dequantizes V itself (the workspace then holds K rows only).
bool prefill_v_in_kernel(int k_dim, int v_dim);
// Stage kernel (Q4 -> fp16 workspace rows of the keys in [p.stage_lo, p.stage_hi)) and/or
// attention kernel (parts: kPrefillStage | kPrefillAttend); p.kd / p.vd / p.nw and the
// tensor maps tmap_kd / tmap_vd describe the workspace.
constexpr int kPrefillStage = 1, kPrefillAttend = 2;
// Workspace rows per block of the stage kernel's grid.
constexpr int kStageRowsHost = 128;
cudaError_t launch_prefill(const DecodeParams& p, int batch, bool paged, bool scale_bf16, int parts,
                           cudaStream_t stream);

// Split size (tokens per CTA chunk), number of chunks and merge mode (1: in-cluster merge)
// for a decode call.
void decode_plan(int batch, int n_kv_heads, int row_groups, int span, int ctas_per_sm, int k_dim,
                 int v_dim, int* chunk, int* n_chunks, int* cluster);
// Largest decode cluster (chunks merged in one thread-block cluster) for a head-dim pair
// on the current device; 0 when cluster merging is unavailable or turned off.
int decode_max_cluster(int k_dim, int v_dim);
// Clusters of `size` decode CTAs that can be resident at once (0: not schedulable).
int decode_active_clusters(int k_dim, int v_dim, int size);
// Resident decode CTAs per SM on the current device for a (k_dim, v_dim) pair.
int decode_ctas_per_sm(int k_dim, int v_dim);

cudaError_t launch_blocks_copy(const BlockCopyParams& p, int n_blocks, cudaStream_t stream);
cudaError_t launch_block_reserve(const BlockListParams& p, cudaStream_t stream);
cudaError_t launch_block_release(const BlockListParams& p, cudaStream_t stream);

}  // namespace am
