// Host-side declarations shared by the kernel translation units and fa_api.cu.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "fa_common.cuh"

namespace fa {

int set_last_error(int code, const char* msg);
// Validation of a backward call's parameters (the checks fa_bwd makes before any work).
int check_bwd_params(const FaBwdParams* p);
// 4-D tensor map over a [B, heads, T, D] tensor (bf16 or fp32): box = one 128-byte panel of
// columns x box_rows rows, 128-byte swizzle.  Rejects misaligned bases and strides.
int make_row_tile_map(CUtensorMap* map, const FaTensor& t, int dtype, int B, int heads, int T, int D, int box_rows,
                      const char* name);

// tcgen05 forward (fa_fwd_sm100.cu)
int fwd_tc_max_stages(int D, int nkv);
cudaError_t launch_fwd_tc(const AttnArgs& a, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                          const CUtensorMap& to, int tile_cfg, cudaStream_t stream);

// tcgen05 backward (fa_bwd_sm100.cu)
int bwd_tc_max_stages(int D, int nq, int G);  // G = H / H_kv query heads per K/V head
int bwd_tc_q_rows(int D);         // q rows per step (the Q / dO tensor-map box height)
cudaError_t launch_bwd_tc(const AttnArgs& a, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                          const CUtensorMap& tdo, const CUtensorMap& tdq, const CUtensorMap& tdk,
                          const CUtensorMap& tdv, cudaStream_t stream);

// generic CUDA-core kernels (fa_simt.cu)
cudaError_t launch_fwd_simt(const AttnArgs& a, int dtype, cudaStream_t stream);
cudaError_t launch_bwd_simt(const AttnArgs& a, int dtype, cudaStream_t stream);

// element-wise helpers (fa_aux.cu)
cudaError_t launch_bwd_preprocess(const AttnArgs& a, int dtype, cudaStream_t stream);
cudaError_t launch_dq_convert(const AttnArgs& a, int dtype, cudaStream_t stream);
cudaError_t launch_lse_merge(int rows, int D, float* o_acc, float* lse_acc, const void* o_part,
                             int64_t o_part_stride, int dtype, const float* lse_part, cudaStream_t stream);

// block masks (fa_blockmask.cu)
cudaError_t launch_create_block_mask(const FaMaskSpec& m, int B, int Tq, int Tkv, int bq, int bkv, int mode,
                                     const FaBlockMaskOut& out, cudaStream_t stream);
cudaError_t launch_tables_from_lists(int num_b, int nq, int nkv, const int32_t* kv_num, const int32_t* kv_idx,
                                     const int32_t* full_num, const int32_t* full_idx, int kv_cap,
                                     const FaBlockMaskOut& out, cudaStream_t stream);

}  // namespace fa
