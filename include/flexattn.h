/*
 * flexattn.h — C ABI of libflexattn.so, the B200 (sm_100a) FlexAttention engine.
 *
 * Every entry point is extern "C", takes plain pointers/sizes and a CUDA stream,
 * returns an int status (FA_OK == 0) and never throws.  fa_last_error() returns a
 * thread-local message for the last failure on the calling thread.  All buffers
 * are owned by the caller; the library allocates no device memory on the hot path
 * (the backward pass takes a caller-provided workspace sized by
 * fa_bwd_workspace_size).
 *
 * Reference interface each entry point replaces (novastar53/pallas-flexattn,
 * paths inside that project):
 *   fa_fwd               <- flash_attention_fwd         src/pallas_flexattn/flash_attn.py:111-165
 *                           (kernel body flash_attention_fwd_kernel, flash_attn.py:59-108)
 *   fa_bwd               <- flash_attention_bwd         src/pallas_flexattn/flash_attn.py:410-461
 *                           (preprocess :168-203, dK/dV :206-310, dQ :313-407)
 *   fa_bwd_preprocess    <- flash_attention_bwd_preprocess flash_attn.py:176-203
 *   fa_create_block_mask <- create_block_mask           src/pallas_flexattn/block_mask.py:54-129
 *   fa_block_tables_from_lists <- BlockMask fields      src/pallas_flexattn/block_mask.py:16-51
 *   fa_lse_merge         <- (no counterpart; combine step of the context-parallel ring)
 *   fa_decode            <- (no counterpart; split-KV decode against a K/V cache)
 */
#ifndef FLEXATTN_H_
#define FLEXATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* fa_stream_t; /* identical to cudaStream_t */

#if defined(__GNUC__)
#define FA_API __attribute__((visibility("default")))
#else
#define FA_API
#endif

/* ------------------------------------------------------------------ status */
enum {
  FA_OK = 0,
  FA_ERR_INVALID = 1,     /* bad argument (shape, stride, pointer, dtype) */
  FA_ERR_UNSUPPORTED = 2, /* valid request this build has no kernel for */
  FA_ERR_CUDA = 3,        /* CUDA runtime/driver error */
  FA_ERR_TIMEOUT = 4,     /* a device-side bounded wait gave up */
};

enum { FA_DTYPE_F32 = 0, FA_DTYPE_BF16 = 1 };

/* Which kernel family runs the attention tiles. */
enum {
  FA_KERNEL_AUTO = 0, /* tcgen05 when the shape allows it, else the SIMT kernel */
  FA_KERNEL_TC = 1,   /* sm_100a tcgen05/TMA/TMEM kernel; error if not applicable */
  FA_KERNEL_SIMT = 2, /* generic CUDA-core kernel (fp32, any D <= 256, any block size) */
};

/* ------------------------------------------------------------------ mask_mod registry
 * A mask is the AND of the enabled predicates on (q_idx, kv_idx):
 *   CAUSAL      q >= kv                                   (mask_mod.py:15-17)
 *   WINDOW      d = q - kv; (left < 0 || d <= left) && (right < 0 || -d <= right)
 *                                                         (mask_mod.py:25-43)
 *   DOCUMENT    doc_q[b][q] == doc_kv[b][kv]              (mask_mod.py:46-59 stub, built here)
 *   TILE_TABLE  table[q / table_block][kv / table_block] != 0
 *   BITMASK     an arbitrary predicate evaluated beforehand into 128 x 128 tiles (the
 *               Python mask_mod callables outside the registry): bit_index[lq/128][lk/128]
 *               is -1 (tile fully masked), -2 (fully allowed) or a slot s whose bits
 *               bits[s][lq%128][(lk%128)/32] >> (lk%32) & 1 hold the predicate, with lq, lk
 *               the LOCAL positions (q - q_offset, kv - kv_offset)
 * No flag set = bidirectional (mask_mod.py:20-22).  Elements with kv >= Tkv are
 * always masked.  Predicates (and the position-dependent score mods) see global
 * positions q + q_offset and kv + kv_offset, so a caller can run one block of a
 * longer sequence (the context-parallel ring does); document ids and the tile
 * table are indexed by global position. */
enum { FA_MASK_CAUSAL = 1, FA_MASK_WINDOW = 2, FA_MASK_DOCUMENT = 4, FA_MASK_TILE_TABLE = 8,
       /* with FA_MASK_DOCUMENT: the ids are non-decreasing along the sequence (contiguous
          documents), so the tcgen05 kernels reduce "same document" to one position interval
          per row instead of testing it per element */
       FA_MASK_DOC_SORTED = 16,
       FA_MASK_BITMASK = 32 };

typedef struct {
  int32_t flags;
  int32_t window_left, window_right; /* -1 = unlimited */
  const int32_t* doc_q;              /* [doc_b, >= q_offset + Tq] device int32 document ids */
  const int32_t* doc_kv;             /* [doc_b, >= kv_offset + Tkv] */
  int64_t doc_stride_b;              /* elements between batches; 0 = shared by all batches */
  const uint8_t* tile_table;         /* [table_rows, table_cols] device bytes, nonzero = keep */
  int32_t table_rows, table_cols, table_block;
  int32_t q_offset, kv_offset;       /* global position of row 0 of q / of k, v */
  const int32_t* bit_index;          /* BITMASK: [bit_rows, bit_cols] device int32 */
  const uint32_t* bits;              /* BITMASK: [slots, 128, 4] device words */
  int32_t bit_rows, bit_cols;        /* ceil(Tq / 128), ceil(Tkv / 128) */
} FaMaskSpec;

/* ------------------------------------------------------------------ score_mod registry
 * Applied in this order to the scaled logit s = scale * q.k:
 *   ALIBI     s += slope[h] * (kv - q)
 *   REL_BIAS  s += bias[h][q - kv + center]
 *   SOFTCAP   s  = cap * tanh(s / cap)   (backward multiplies by 1 - tanh^2)
 * with global positions q, kv (see FaMaskSpec offsets). */
enum { FA_SCORE_ALIBI = 1, FA_SCORE_SOFTCAP = 2, FA_SCORE_REL_BIAS = 4 };

typedef struct {
  int32_t flags;
  float softcap;
  const float* alibi_slopes; /* [H] device fp32 */
  const float* rel_bias;     /* [H or 1, L] device fp32, L covers every q - kv + center used */
  int64_t rel_bias_stride_h; /* 0 = one table for all heads */
  int32_t rel_bias_center;   /* table index of q == kv; <= 0 means Tkv - 1 */
} FaScoreSpec;

/* ------------------------------------------------------------------ block tables
 * FlexAttention-style sparse tile tables.  For q block i, the kv blocks to visit
 * with the mask applied are kv_indices[i][0 .. kv_num_blocks[i]) ("partial"), and
 * the ones visited without evaluating the mask are full_kv_indices[i][0 ..
 * full_kv_num_blocks[i]) ("full").  Blocks in neither list are skipped.  The q_*
 * tables are the transpose (per kv block), used by the backward pass.  Tables
 * carry a leading [num_b, num_h] index; a dimension of 1 broadcasts. */
typedef struct {
  int32_t block_q, block_kv; /* tile sizes the tables describe */
  int32_t nq, nkv;           /* ceil(Tq / block_q), ceil(Tkv / block_kv) */
  int32_t num_b, num_h;      /* 1 or B, 1 or H */
  const int32_t* kv_num_blocks;      /* [num_b, num_h, nq] */
  const int32_t* kv_indices;         /* [num_b, num_h, nq, kv_cap] */
  const int32_t* full_kv_num_blocks; /* may be NULL */
  const int32_t* full_kv_indices;
  int32_t kv_cap;
  const int32_t* q_num_blocks;      /* [num_b, num_h, nkv]; required by fa_bwd */
  const int32_t* q_indices;         /* [num_b, num_h, nkv, q_cap] */
  const int32_t* full_q_num_blocks; /* may be NULL */
  const int32_t* full_q_indices;
  int32_t q_cap;
} FaBlockTables;

/* A [B, H, T, D] tensor whose last dimension is contiguous. Strides in elements. */
typedef struct {
  void* ptr;
  int64_t stride_b, stride_h, stride_t;
} FaTensor;

/* Launch shape of the tcgen05 forward (FaFwdParams.tile_cfg), the measured autotuner's
 * choices besides the pipeline depth.  Bits 0-1: Q tiles per CTA; bits 2-3: softmax schedule
 * of the two sub-tiles; bits 4-5: softmax warps per row; bit 6: kv halves.  0 in a field = the
 * launcher's per-launch choice. */
enum {
  FA_TILE_Q2 = 1,                 /* two 128-row Q tiles per CTA sharing each K/V tile load */
  FA_TILE_Q1 = 2,                 /* one Q tile per CTA (twice the CTAs; for small grids) */
  FA_TILE_HEADS2 = 3,             /* one Q tile of two heads per CTA: both walk the same kv list
                                     (irregular sparse masks); H must be even */
  FA_TILE_SOFTMAX_CONCURRENT = 4, /* both softmax warpgroups run at once */
  FA_TILE_SOFTMAX_TURNS = 8,      /* strict turns per kv tile (no score_mod only) */
  FA_TILE_ROWS_SPLIT = 16,        /* bits 4-5: each softmax row shared by two warps (64 columns each) */
  FA_TILE_ROWS_WHOLE = 32,        /*           one warp per row (128 columns) */
  FA_TILE_KV_HALVES = 64,         /* bit 6: one Q tile per CTA, its kv list split over the two
                                     sub-tiles and merged at the end (small grids, long rows);
                                     shape bits 0-1 must be 0, rows whole */
};

typedef struct {
  int32_t dtype;            /* FA_DTYPE_BF16 or FA_DTYPE_F32; q/k/v/o share it */
  int32_t B, H, H_kv;       /* H_kv divides H (grouped-query attention when < H) */
  int32_t Tq, Tkv, D;
  FaTensor q, k, v, o;
  float* lse;               /* [B, H, Tq] fp32 natural-log logsumexp; contiguous */
  float scale;              /* softmax scale (1/sqrt(D) in the reference) */
  FaMaskSpec mask;
  FaScoreSpec score;
  FaBlockTables blocks;
  int32_t kernel;           /* FA_KERNEL_* */
  int32_t num_stages;       /* K/V entries in flight in the tcgen05 forward (each = K + V tile);
                               0 = as many as shared memory holds */
  int32_t* status;          /* optional device int32: nonzero after a device-side timeout */
  int32_t tile_cfg;         /* FA_TILE_* launch shape of the tcgen05 forward; 0 = chosen per launch */
} FaFwdParams;

typedef struct {
  int32_t dtype;
  int32_t B, H, H_kv;       /* H_kv divides H; dk / dv have H_kv heads (sum over each group) */
  int32_t Tq, Tkv, D;
  FaTensor q, k, v, o, dout;
  FaTensor dq, dk, dv;
  const float* lse;         /* [B, H, Tq] from fa_fwd */
  float scale;
  FaMaskSpec mask;
  FaScoreSpec score;
  FaBlockTables blocks;
  int32_t kernel;
  int32_t num_stages;       /* Q/dO tiles in flight in the tcgen05 backward; 0 = default (2) */
  int32_t* status;
  int32_t tile_cfg;         /* reserved for launch-shape choices of the backward; pass 0 */
} FaBwdParams;

/* ------------------------------------------------------------------ entry points */
FA_API const char* fa_version(void);
FA_API const char* fa_last_error(void);

/* Forward: o, lse <- attention(q, k, v).  Rows with no unmasked key get o = 0 and
 * lse = -inf. */
FA_API int fa_fwd(const FaFwdParams* p, fa_stream_t stream);

/* delta[b,h,t] = sum_d o*dout (fp32) and zero the fp32 dQ accumulator. */
FA_API int fa_bwd_preprocess(const FaBwdParams* p, float* delta, float* dq_accum, fa_stream_t stream);

/* Bytes of device workspace fa_bwd needs (delta + fp32 dQ accumulator). */
FA_API int fa_bwd_workspace_size(const FaBwdParams* p, size_t* bytes);

/* Backward: dq, dk, dv from (q, k, v, o, lse, dout).  Runs preprocess, the fused
 * dK/dV/dQ kernel and the dQ conversion. */
FA_API int fa_bwd(const FaBwdParams* p, void* workspace, size_t workspace_bytes, fa_stream_t stream);

/* Backward like fa_bwd, but allocation-free: the workspace is a static device array of
 * FA_NOALLOC_SCRATCH_BYTES inside the library instead of caller memory.  No counterpart
 * in the reference (its backward gets scratch from the XLA runtime); it serves hosts that
 * hold device pointers but no device allocator, e.g. a cgo/JNI/ctypes binding running
 * inside another runtime's memory pool, where a cudaMalloc bypasses the pool and can
 * fail once the pool has reserved most of the HBM.
 * - Limit: a shape whose fa_bwd_workspace_size exceeds FA_NOALLOC_SCRATCH_BYTES returns
 *   FA_ERR_UNSUPPORTED before anything runs (use fa_bwd for it).
 * - The scratch's address belongs to a CUDA context: the first call in each context (a
 *   device's primary context, or one the host created with cuCtxCreate), with that context
 *   current, resolves it and loads the kernels; make that call before any stream capture.
 * - Calls that overlap on one device share the scratch and race: serialise them. */
#define FA_NOALLOC_SCRATCH_BYTES ((size_t)64 << 20)
FA_API int fa_bwd_noalloc(const FaBwdParams* p, fa_stream_t stream);

/* Block-mask construction on the GPU. */
enum {
  FA_BLOCK_MASK_EXACT = 0, /* tile listed iff any element is unmasked; "full" iff all are */
  FA_BLOCK_MASK_REF9 = 1,  /* the reference's 3x3 sampling rule; every listed tile is partial */
};

typedef struct {
  int32_t num_b, nq, nkv;        /* outputs are [num_b, 1, ...]; num_b = 1 unless the mask
                                    depends on the batch (document ids with doc_stride_b != 0) */
  uint8_t* tile_class;           /* [num_b, nq, nkv]: 0 skip, 1 partial, 2 full */
  int32_t* kv_num_blocks;        /* [num_b, nq] */
  int32_t* kv_indices;           /* [num_b, nq, nkv], rows padded with -1 */
  int32_t* full_kv_num_blocks;   /* [num_b, nq] */
  int32_t* full_kv_indices;      /* [num_b, nq, nkv] */
  int32_t* q_num_blocks;         /* [num_b, nkv] */
  int32_t* q_indices;            /* [num_b, nkv, nq] */
  int32_t* full_q_num_blocks;    /* [num_b, nkv] */
  int32_t* full_q_indices;       /* [num_b, nkv, nq] */
} FaBlockMaskOut;

FA_API int fa_create_block_mask(const FaMaskSpec* mask, int32_t B, int32_t Tq, int32_t Tkv, int32_t block_q,
                         int32_t block_kv, int32_t mode, FaBlockMaskOut* out, fa_stream_t stream);

/* Rebuild tile_class and all four table pairs of `out` from row lists (partial
 * kv_num_blocks/kv_indices with row length kv_cap, optional full lists). */
FA_API int fa_block_tables_from_lists(int32_t num_b, int32_t nq, int32_t nkv, const int32_t* kv_num_blocks,
                               const int32_t* kv_indices, const int32_t* full_kv_num_blocks,
                               const int32_t* full_kv_indices, int32_t kv_cap, FaBlockMaskOut* out,
                               fa_stream_t stream);

/* Combine two partial attention results over disjoint key sets, in place into
 * (o_acc, lse_acc):  lse = logaddexp(lse_acc, lse_part);
 *                    o   = o_acc*exp(lse_acc-lse) + o_part*exp(lse_part-lse).
 * o_acc is fp32 [rows, D]; o_part is dtype [rows, D] with row stride o_part_stride. */
FA_API int fa_lse_merge(int32_t rows, int32_t D, float* o_acc, float* lse_acc, const void* o_part,
                 int64_t o_part_stride, int32_t o_part_dtype, const float* lse_part, fa_stream_t stream);

/* ------------------------------------------------------------------ decode (split-KV)
 * Attention of a few new query tokens per sequence against a K/V cache.  Batch b holds
 * kv_lens[b] valid cache positions (all Tkv when kv_lens is NULL); its Tq query rows are
 * the last Tq positions of that sequence: row i sits at global position
 * kv_lens[b] - Tq + i, which the mask and score mods see (causal = keys up to the row's
 * own position).  The cache is cut into num_splits chunks handled by separate CTAs (one
 * per chunk, batch and K/V head, covering every query head of the group), and a second
 * kernel merges the chunks' (o, lse).  bf16 runs on the tensor cores (tcgen05), fp32 on
 * CUDA cores.  Supported: D in {64, 128, 256}, H / H_kv * Tq <= 128 (bf16) or <= 64 (fp32),
 * mask flags CAUSAL / WINDOW, score flags ALIBI / SOFTCAP.  No counterpart in the
 * reference. */
typedef struct {
  int32_t dtype;            /* FA_DTYPE_BF16 or FA_DTYPE_F32 */
  int32_t B, H, H_kv, Tq, Tkv, D;
  FaTensor q, k, v, o;      /* q, o [B, H, Tq, D]; k, v [B, H_kv, Tkv, D] (the cache) */
  float* lse;               /* [B, H, Tq] fp32 natural-log logsumexp */
  const int32_t* kv_lens;   /* [B] device int32 valid cache lengths (Tq <= len <= Tkv), or NULL */
  float scale;
  FaMaskSpec mask;          /* q_offset / kv_offset must be 0 (positions come from kv_lens) */
  FaScoreSpec score;
  int32_t num_splits;       /* cache chunks per (b, K/V head); 0 = chosen from the shape */
  int32_t* status;          /* optional, as in FaFwdParams */
} FaDecodeParams;

/* Bytes of device workspace fa_decode needs (the chunks' partial o and lse). */
FA_API int fa_decode_workspace_size(const FaDecodeParams* p, size_t* bytes);
FA_API int fa_decode(const FaDecodeParams* p, void* workspace, size_t workspace_bytes, fa_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* FLEXATTN_H_ */
