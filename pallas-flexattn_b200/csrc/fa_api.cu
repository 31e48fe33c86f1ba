// C-ABI entry points of libflexattn.so (declared in include/flexattn.h): argument
// validation, TMA tensor-map encoding and kernel dispatch.  No exception crosses
// this boundary; failures return a status code and set a thread-local message.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "fa_internal.h"
#include "flexattn.h"

namespace fa {
namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(FA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 4-D map over a bf16 [B, heads, T, D] tensor; box = 64 columns x box_rows rows, 128-byte swizzle.
int make_bf16_map(CUtensorMap* map, const FaTensor& t, int B, int heads, int T, int D, const char* name,
                  int box_rows = 128) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(FA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)heads, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)t.stride_t * 2, (cuuint64_t)t.stride_h * 2, (cuuint64_t)t.stride_b * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, t.ptr, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FA_ERR_INVALID, "tensor map for %s rejected (CUresult %d)", name, (int)r);
  return FA_OK;
}

// 3-D map over the fp32 dQ accumulator [B*H, Tq, D]; box = 32 columns x 32 rows, 128-byte
// swizzle (the layout the drain warps stage in shared memory).  Rows past Tq are out of
// bounds, so reduce-adds of a partial last tile never touch the next head.
int make_dq_accum_map(CUtensorMap* map, float* base, int BH, int Tq, int D) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(FA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)Tq, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)D * 4, (cuuint64_t)Tq * D * 4};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FA_ERR_INVALID, "tensor map for the dQ accumulator rejected (CUresult %d)", (int)r);
  return FA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_tensor(const FaTensor& t, const char* name, int elem) {
  if (!t.ptr) return fail(FA_ERR_INVALID, "%s is NULL", name);
  if (t.stride_b < 0 || t.stride_h < 0 || t.stride_t < 0) return fail(FA_ERR_INVALID, "%s has negative stride", name);
  (void)elem;
  return FA_OK;
}

bool tc_tensor_ok(const FaTensor& t) {
  return aligned16(t.ptr) && (t.stride_t * 2) % 16 == 0 && (t.stride_h * 2) % 16 == 0 &&
         (t.stride_b * 2) % 16 == 0;
}

int check_common(int dtype, int B, int H, int Hkv, int Tq, int Tkv, int D, const FaBlockTables& bt,
                 const FaMaskSpec& m, const FaScoreSpec& s) {
  if (dtype != FA_DTYPE_BF16 && dtype != FA_DTYPE_F32) return fail(FA_ERR_INVALID, "unknown dtype %d", dtype);
  if (B <= 0 || H <= 0 || Hkv <= 0 || Tq <= 0 || Tkv <= 0 || D <= 0)
    return fail(FA_ERR_INVALID, "non-positive shape B=%d H=%d H_kv=%d Tq=%d Tkv=%d D=%d", B, H, Hkv, Tq, Tkv, D);
  if (H % Hkv != 0) return fail(FA_ERR_INVALID, "H=%d is not a multiple of H_kv=%d", H, Hkv);
  if (D > 256 || D % 8 != 0) return fail(FA_ERR_UNSUPPORTED, "head dim %d (need a multiple of 8, <= 256)", D);
  if (bt.block_q <= 0 || bt.block_kv <= 0) return fail(FA_ERR_INVALID, "block sizes must be positive");
  if (bt.nq != (Tq + bt.block_q - 1) / bt.block_q || bt.nkv != (Tkv + bt.block_kv - 1) / bt.block_kv)
    return fail(FA_ERR_INVALID, "block tables (nq=%d, nkv=%d) do not match Tq=%d/Tkv=%d with blocks %dx%d", bt.nq,
                bt.nkv, Tq, Tkv, bt.block_q, bt.block_kv);
  if (!(bt.num_b == 1 || bt.num_b == B) || !(bt.num_h == 1 || bt.num_h == H))
    return fail(FA_ERR_INVALID, "block tables num_b=%d num_h=%d must be 1 or B/H", bt.num_b, bt.num_h);
  if (!bt.kv_num_blocks && !bt.full_kv_num_blocks) return fail(FA_ERR_INVALID, "no kv block tables");
  if (bt.kv_num_blocks && !bt.kv_indices) return fail(FA_ERR_INVALID, "kv_indices is NULL");
  if (bt.full_kv_num_blocks && !bt.full_kv_indices) return fail(FA_ERR_INVALID, "full_kv_indices is NULL");
  if (bt.kv_cap <= 0) return fail(FA_ERR_INVALID, "kv_cap must be positive");
  if ((m.flags & FA_MASK_DOCUMENT) && (!m.doc_q || !m.doc_kv))
    return fail(FA_ERR_INVALID, "document mask without document ids");
  if ((m.flags & FA_MASK_TILE_TABLE) && (!m.tile_table || m.table_block <= 0 || m.table_cols <= 0))
    return fail(FA_ERR_INVALID, "tile-table mask without a table");
  // the kernels index the table by position, up to the last (padded) 128-row tile
  if ((m.flags & FA_MASK_TILE_TABLE) &&
      ((int64_t)m.table_rows * m.table_block < (int64_t)m.q_offset + (Tq + 127) / 128 * 128 ||
       (int64_t)m.table_cols * m.table_block < (int64_t)m.kv_offset + (Tkv + 127) / 128 * 128))
    return fail(FA_ERR_INVALID, "tile table of %d x %d cells of %d does not cover %d x %d positions (rounded up "
                "to 128)", m.table_rows, m.table_cols, m.table_block, m.q_offset + Tq, m.kv_offset + Tkv);
  if (m.flags & ~(FA_MASK_CAUSAL | FA_MASK_WINDOW | FA_MASK_DOCUMENT | FA_MASK_TILE_TABLE | FA_MASK_DOC_SORTED |
                  FA_MASK_BITMASK))
    return fail(FA_ERR_INVALID, "unknown mask flags 0x%x", m.flags);
  if ((m.flags & FA_MASK_BITMASK) &&
      (!m.bit_index || !m.bits || m.bit_rows < (Tq + 127) / 128 || m.bit_cols < (Tkv + 127) / 128))
    return fail(FA_ERR_INVALID, "bitmask mask without tables covering %d x %d positions", Tq, Tkv);
  if ((m.flags & FA_MASK_DOC_SORTED) && !(m.flags & FA_MASK_DOCUMENT))
    return fail(FA_ERR_INVALID, "FA_MASK_DOC_SORTED needs FA_MASK_DOCUMENT");
  if (s.flags & ~(FA_SCORE_ALIBI | FA_SCORE_SOFTCAP | FA_SCORE_REL_BIAS))
    return fail(FA_ERR_INVALID, "unknown score flags 0x%x", s.flags);
  if ((s.flags & FA_SCORE_ALIBI) && !s.alibi_slopes) return fail(FA_ERR_INVALID, "ALiBi without slopes");
  if ((s.flags & FA_SCORE_REL_BIAS) && !s.rel_bias) return fail(FA_ERR_INVALID, "relative bias without a table");
  if ((s.flags & FA_SCORE_SOFTCAP) && !(s.softcap > 0.f)) return fail(FA_ERR_INVALID, "softcap must be > 0");
  return FA_OK;
}

AttnArgs base_args(int B, int H, int Hkv, int Tq, int Tkv, int D, float scale, const FaMaskSpec& m,
                   const FaScoreSpec& s, const FaBlockTables& bt, int* status) {
  AttnArgs a;
  memset(&a, 0, sizeof(a));
  a.B = B; a.H = H; a.Hkv = Hkv; a.Tq = Tq; a.Tkv = Tkv; a.D = D;
  a.scale = scale; a.mask = m; a.score = s; a.bt = bt; a.status = status;
  return a;
}

}  // namespace

// Sets the thread's fa_last_error message from another translation unit; returns `code`.
int set_last_error(int code, const char* msg) { return fail(code, "%s", msg); }

int make_row_tile_map(CUtensorMap* map, const FaTensor& t, int dtype, int B, int heads, int T, int D, int box_rows,
                      const char* name) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(FA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const int es = dtype == FA_DTYPE_F32 ? 4 : 2;
  if (!aligned16(t.ptr) || (t.stride_t * es) % 16 || (t.stride_h * es) % 16 || (t.stride_b * es) % 16)
    return fail(FA_ERR_INVALID, "%s: base address and strides must be multiples of 16 bytes", name);
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)heads, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)t.stride_t * es, (cuuint64_t)t.stride_h * es, (cuuint64_t)t.stride_b * es};
  cuuint32_t box[4] = {(cuuint32_t)(128 / es), (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, es == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, t.ptr, dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FA_ERR_INVALID, "tensor map for %s rejected (CUresult %d)", name, (int)r);
  return FA_OK;
}

}  // namespace fa

using namespace fa;

extern "C" {

const char* fa_version(void) { return "flexattn-b200 0.1.0 (sm_100a)"; }

const char* fa_last_error(void) { return g_err; }

int fa_fwd(const FaFwdParams* p, fa_stream_t stream) {
  if (!p) return fail(FA_ERR_INVALID, "params is NULL");
  int rc = check_common(p->dtype, p->B, p->H, p->H_kv, p->Tq, p->Tkv, p->D, p->blocks, p->mask, p->score);
  if (rc) return rc;
  if ((rc = check_tensor(p->q, "q", 0)) || (rc = check_tensor(p->k, "k", 0)) || (rc = check_tensor(p->v, "v", 0)) ||
      (rc = check_tensor(p->o, "o", 0)))
    return rc;
  if (!p->lse) return fail(FA_ERR_INVALID, "lse is NULL");
  AttnArgs a = base_args(p->B, p->H, p->H_kv, p->Tq, p->Tkv, p->D, p->scale, p->mask, p->score, p->blocks, p->status);
  a.q = p->q; a.k = p->k; a.v = p->v; a.o = p->o; a.lse = p->lse;

  const bool tc_ok = p->dtype == FA_DTYPE_BF16 && (p->D == 64 || p->D == 128) && p->blocks.block_q == 128 &&
                     p->blocks.block_kv == 128 && tc_tensor_ok(p->q) && tc_tensor_ok(p->k) && tc_tensor_ok(p->v) &&
                     tc_tensor_ok(p->o) && fwd_tc_max_stages(p->D, p->blocks.nkv) >= 2;
  int kernel = p->kernel;
  if (kernel == FA_KERNEL_AUTO) kernel = tc_ok ? FA_KERNEL_TC : FA_KERNEL_SIMT;
  if (kernel == FA_KERNEL_TC) {
    if (!tc_ok)
      return fail(FA_ERR_UNSUPPORTED,
                  "tcgen05 forward needs bf16, D in {64,128}, 128x128 block tables and 16-byte aligned rows");
    if ((p->tile_cfg & ~127) || (p->tile_cfg & 48) == 48 ||
        ((p->tile_cfg & FA_TILE_KV_HALVES) && ((p->tile_cfg & 3) || (p->tile_cfg & 48) == FA_TILE_ROWS_SPLIT)))
      return fail(FA_ERR_INVALID, "unknown or conflicting tile_cfg bits 0x%x", p->tile_cfg);
    if ((p->tile_cfg & 3) == FA_TILE_HEADS2 && p->H % 2)
      return fail(FA_ERR_INVALID, "FA_TILE_HEADS2 pairs heads: H=%d must be even", p->H);
    // num_stages counts K/V entries in flight (the reference's pipelining depth); each
    // entry takes two ring slots (K and V).  0 = as deep as shared memory allows.
    const int max_ns = fwd_tc_max_stages(p->D, p->blocks.nkv);
    int ns = p->num_stages > 0 ? 2 * p->num_stages : max_ns;
    if (ns < 2) ns = 2;
    if (ns > max_ns) ns = max_ns;
    a.num_stages = ns;
    CUtensorMap tq, tk, tv, to;
    if ((rc = make_bf16_map(&tq, p->q, p->B, p->H, p->Tq, p->D, "q")) ||
        (rc = make_bf16_map(&tk, p->k, p->B, p->H_kv, p->Tkv, p->D, "k")) ||
        (rc = make_bf16_map(&tv, p->v, p->B, p->H_kv, p->Tkv, p->D, "v")) ||
        (rc = make_bf16_map(&to, p->o, p->B, p->H, p->Tq, p->D, "o")))
      return rc;
    cudaError_t e = launch_fwd_tc(a, tq, tk, tv, to, p->tile_cfg, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "fa_fwd (tcgen05)");
    return FA_OK;
  }
  if (kernel != FA_KERNEL_SIMT) return fail(FA_ERR_INVALID, "unknown kernel selector %d", kernel);
  cudaError_t e = launch_fwd_simt(a, p->dtype, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "fa_fwd (simt)");
  return FA_OK;
}

extern "C++" {
namespace fa {
// Argument validation shared by fa_bwd, fa_bwd_preprocess and fa_bwd_noalloc.
int check_bwd_params(const FaBwdParams* p) {
  if (!p) return fail(FA_ERR_INVALID, "params is NULL");
  int rc = check_common(p->dtype, p->B, p->H, p->H_kv, p->Tq, p->Tkv, p->D, p->blocks, p->mask, p->score);
  if (rc) return rc;
  if ((rc = check_tensor(p->q, "q", 0)) || (rc = check_tensor(p->k, "k", 0)) || (rc = check_tensor(p->v, "v", 0)) ||
      (rc = check_tensor(p->o, "o", 0)) || (rc = check_tensor(p->dout, "dout", 0)) ||
      (rc = check_tensor(p->dq, "dq", 0)) || (rc = check_tensor(p->dk, "dk", 0)) || (rc = check_tensor(p->dv, "dv", 0)))
    return rc;
  if (!p->lse) return fail(FA_ERR_INVALID, "lse is NULL");
  if (!p->blocks.q_num_blocks && !p->blocks.full_q_num_blocks)
    return fail(FA_ERR_INVALID, "backward needs the transposed (q_*) block tables");
  if (p->blocks.q_num_blocks && !p->blocks.q_indices) return fail(FA_ERR_INVALID, "q_indices is NULL");
  if (p->blocks.full_q_num_blocks && !p->blocks.full_q_indices) return fail(FA_ERR_INVALID, "full_q_indices is NULL");
  if (p->blocks.q_cap <= 0) return fail(FA_ERR_INVALID, "q_cap must be positive");
  return FA_OK;
}
}  // namespace fa
}  // extern "C++"

static size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

static int pad128(int t) { return (t + 127) / 128 * 128; }

// Workspace: delta [B*H, Tq_pad] | lse2 [B*H, Tq_pad] | dq_accum [B*H, Tq, D], fp32 (sized
// B*H*Tq_pad*D: the preprocess kernel zeroes it per padded row).
int fa_bwd_workspace_size(const FaBwdParams* p, size_t* bytes) {
  if (!p || !bytes) return fail(FA_ERR_INVALID, "NULL argument");
  const size_t prow = (size_t)p->B * p->H * pad128(p->Tq);
  const size_t rows = prow;
  *bytes = 2 * round_up(prow * sizeof(float), 256) + round_up(rows * p->D * sizeof(float), 256);
  return FA_OK;
}

int fa_bwd_preprocess(const FaBwdParams* p, float* delta, float* dq_accum, fa_stream_t stream) {
  int rc = check_bwd_params(p);
  if (rc) return rc;
  if (!delta || !dq_accum) return fail(FA_ERR_INVALID, "delta / dq_accum is NULL");
  AttnArgs a = base_args(p->B, p->H, p->H_kv, p->Tq, p->Tkv, p->D, p->scale, p->mask, p->score, p->blocks, p->status);
  a.o = p->o; a.dout = p->dout; a.delta = delta; a.dq_accum = dq_accum;
  a.Tq_pad = p->Tq;  // public form: delta is [B*H, Tq], no log2 logsumexp
  a.lse2 = nullptr;
  cudaError_t e = launch_bwd_preprocess(a, p->dtype, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "fa_bwd_preprocess");
  return FA_OK;
}

int fa_bwd(const FaBwdParams* p, void* workspace, size_t workspace_bytes, fa_stream_t stream) {
  int rc = check_bwd_params(p);
  if (rc) return rc;
  size_t need = 0;
  fa_bwd_workspace_size(p, &need);
  if (!workspace || workspace_bytes < need)
    return fail(FA_ERR_INVALID, "workspace too small (%zu < %zu bytes)", workspace_bytes, need);
  if (!aligned16(workspace)) return fail(FA_ERR_INVALID, "workspace must be 16-byte aligned");
  const size_t prow_bytes = round_up((size_t)p->B * p->H * pad128(p->Tq) * 4, 256);
  char* ws = reinterpret_cast<char*>(workspace);

  AttnArgs a = base_args(p->B, p->H, p->H_kv, p->Tq, p->Tkv, p->D, p->scale, p->mask, p->score, p->blocks, p->status);
  a.q = p->q; a.k = p->k; a.v = p->v; a.o = p->o; a.dout = p->dout;
  a.dq = p->dq; a.dk = p->dk; a.dv = p->dv;
  a.lse_in = p->lse;
  a.Tq_pad = pad128(p->Tq);
  a.delta = reinterpret_cast<float*>(ws);
  a.lse2 = reinterpret_cast<float*>(ws + prow_bytes);
  a.dq_accum = reinterpret_cast<float*>(ws + 2 * prow_bytes);

  cudaError_t e = launch_bwd_preprocess(a, p->dtype, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "fa_bwd preprocess");

  const bool tc_ok = p->dtype == FA_DTYPE_BF16 && (p->D == 64 || p->D == 128) && p->blocks.block_q == 128 &&
                     p->blocks.block_kv == 128 && tc_tensor_ok(p->q) && tc_tensor_ok(p->k) && tc_tensor_ok(p->v) &&
                     tc_tensor_ok(p->dout) && tc_tensor_ok(p->dk) && tc_tensor_ok(p->dv) &&
                     bwd_tc_max_stages(p->D, p->blocks.nq, p->H / p->H_kv) >= 1;
  int kernel = p->kernel;
  if (kernel == FA_KERNEL_AUTO) kernel = tc_ok ? FA_KERNEL_TC : FA_KERNEL_SIMT;
  if (kernel == FA_KERNEL_TC) {
    if (!tc_ok)
      return fail(FA_ERR_UNSUPPORTED,
                  "tcgen05 backward needs bf16, D in {64,128}, 128x128 block tables and 16-byte aligned rows");
    const int max_ns = bwd_tc_max_stages(p->D, p->blocks.nq, p->H / p->H_kv);
    int ns = p->num_stages > 0 ? p->num_stages : 2;
    if (ns > max_ns) ns = max_ns;
    a.num_stages = ns;
    CUtensorMap tq, tk, tv, tdo, tdq, tdk, tdv;
    const int qrows = bwd_tc_q_rows(p->D);
    if ((rc = make_bf16_map(&tq, p->q, p->B, p->H, p->Tq, p->D, "q", qrows)) ||
        (rc = make_bf16_map(&tk, p->k, p->B, p->H_kv, p->Tkv, p->D, "k")) ||
        (rc = make_bf16_map(&tv, p->v, p->B, p->H_kv, p->Tkv, p->D, "v")) ||
        (rc = make_bf16_map(&tdo, p->dout, p->B, p->H, p->Tq, p->D, "dout", qrows)) ||
        (rc = make_dq_accum_map(&tdq, a.dq_accum, p->B * p->H, p->Tq, p->D)) ||
        (rc = make_bf16_map(&tdk, p->dk, p->B, p->H_kv, p->Tkv, p->D, "dk")) ||
        (rc = make_bf16_map(&tdv, p->dv, p->B, p->H_kv, p->Tkv, p->D, "dv")))
      return rc;
    e = launch_bwd_tc(a, tq, tk, tv, tdo, tdq, tdk, tdv, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "fa_bwd (tcgen05)");
  } else if (kernel == FA_KERNEL_SIMT) {
    e = launch_bwd_simt(a, p->dtype, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "fa_bwd (simt)");
  } else {
    return fail(FA_ERR_INVALID, "unknown kernel selector %d", kernel);
  }
  e = launch_dq_convert(a, p->dtype, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "fa_bwd dq convert");
  return FA_OK;
}

int fa_create_block_mask(const FaMaskSpec* mask, int32_t B, int32_t Tq, int32_t Tkv, int32_t block_q,
                         int32_t block_kv, int32_t mode, FaBlockMaskOut* out, fa_stream_t stream) {
  if (!mask || !out) return fail(FA_ERR_INVALID, "NULL argument");
  if (B <= 0 || Tq <= 0 || Tkv <= 0 || block_q <= 0 || block_kv <= 0)
    return fail(FA_ERR_INVALID, "non-positive size");
  if (mode != FA_BLOCK_MASK_EXACT && mode != FA_BLOCK_MASK_REF9) return fail(FA_ERR_INVALID, "unknown mode %d", mode);
  const int nq = (Tq + block_q - 1) / block_q, nkv = (Tkv + block_kv - 1) / block_kv;
  if (out->nq != nq || out->nkv != nkv) return fail(FA_ERR_INVALID, "out nq/nkv (%d,%d) != (%d,%d)", out->nq, out->nkv, nq, nkv);
  const int need_b = ((mask->flags & FA_MASK_DOCUMENT) && mask->doc_stride_b != 0) ? B : 1;
  if (out->num_b != need_b) return fail(FA_ERR_INVALID, "out num_b=%d, this mask needs %d", out->num_b, need_b);
  if ((mask->flags & FA_MASK_DOCUMENT) && (!mask->doc_q || !mask->doc_kv))
    return fail(FA_ERR_INVALID, "document mask without document ids");
  if ((mask->flags & FA_MASK_TILE_TABLE) && (!mask->tile_table || mask->table_block <= 0))
    return fail(FA_ERR_INVALID, "tile-table mask without a table");
  if ((mask->flags & FA_MASK_BITMASK) && (!mask->bit_index || !mask->bits || mask->bit_rows < (Tq + 127) / 128 ||
                                          mask->bit_cols < (Tkv + 127) / 128))
    return fail(FA_ERR_INVALID, "bitmask mask without tables covering %d x %d positions", Tq, Tkv);
  if (!out->tile_class || !out->kv_num_blocks || !out->kv_indices || !out->full_kv_num_blocks ||
      !out->full_kv_indices || !out->q_num_blocks || !out->q_indices || !out->full_q_num_blocks || !out->full_q_indices)
    return fail(FA_ERR_INVALID, "an output table pointer is NULL");
  cudaError_t e = launch_create_block_mask(*mask, B, Tq, Tkv, block_q, block_kv, mode, *out, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "fa_create_block_mask");
  return FA_OK;
}

int fa_block_tables_from_lists(int32_t num_b, int32_t nq, int32_t nkv, const int32_t* kv_num_blocks,
                               const int32_t* kv_indices, const int32_t* full_kv_num_blocks,
                               const int32_t* full_kv_indices, int32_t kv_cap, FaBlockMaskOut* out,
                               fa_stream_t stream) {
  if (!out || num_b <= 0 || nq <= 0 || nkv <= 0 || kv_cap <= 0) return fail(FA_ERR_INVALID, "bad argument");
  if (!kv_num_blocks && !full_kv_num_blocks) return fail(FA_ERR_INVALID, "no row lists");
  if ((kv_num_blocks && !kv_indices) || (full_kv_num_blocks && !full_kv_indices))
    return fail(FA_ERR_INVALID, "counts without indices");
  if (out->num_b != num_b || out->nq != nq || out->nkv != nkv) return fail(FA_ERR_INVALID, "out shape mismatch");
  cudaError_t e = launch_tables_from_lists(num_b, nq, nkv, kv_num_blocks, kv_indices, full_kv_num_blocks,
                                           full_kv_indices, kv_cap, *out, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "fa_block_tables_from_lists");
  return FA_OK;
}

int fa_lse_merge(int32_t rows, int32_t D, float* o_acc, float* lse_acc, const void* o_part, int64_t o_part_stride,
                 int32_t o_part_dtype, const float* lse_part, fa_stream_t stream) {
  if (rows < 0 || D <= 0 || !o_acc || !lse_acc || !o_part || !lse_part) return fail(FA_ERR_INVALID, "bad argument");
  if (o_part_dtype != FA_DTYPE_BF16 && o_part_dtype != FA_DTYPE_F32) return fail(FA_ERR_INVALID, "bad dtype");
  if (rows == 0) return FA_OK;
  cudaError_t e = launch_lse_merge(rows, D, o_acc, lse_acc, o_part, o_part_stride, o_part_dtype, lse_part,
                                   (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "fa_lse_merge");
  return FA_OK;
}

}  // extern "C"
