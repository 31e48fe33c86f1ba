// Device-side building blocks shared by every FlexAttention kernel: the mask_mod
// and score_mod functor registry, block-table addressing and kernel argument packs.
#pragma once
#include <cuda_bf16.h>
#include <cstdint>

#include "flexattn.h"

namespace fa {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Compile-time score_mod selection for the hot kernels.  SC_GENERAL evaluates the
// runtime flags (any combination of ALiBi, relative bias and softcap).
enum ScoreKind : int { SC_NONE = 0, SC_ALIBI = 1, SC_SOFTCAP = 2, SC_GENERAL = 3 };

__host__ __device__ inline int score_kind_of(int flags) {
  if (flags == 0) return SC_NONE;
  if (flags == FA_SCORE_ALIBI) return SC_ALIBI;
  if (flags == FA_SCORE_SOFTCAP) return SC_SOFTCAP;
  return SC_GENERAL;
}

// Per-(b,h) constants of the score_mod, prepared once per CTA.  All results are
// returned in the log2 domain (natural logit * log2(e)) because the kernels use ex2.
struct ScoreCtx {
  int flags;
  float scale;       // softmax scale
  float k_log2;      // scale * log2(e)
  float slope_log2;  // alibi slope[h] * log2(e)
  float slope;       // alibi slope[h]
  float cap;         // softcap
  float cap_log2;    // cap * log2(e)
  float inv_cap;     // 1 / cap
  const float* bias; // relative-bias row of head h, indexed q - kv + bias_off
  int bias_off;
};

__device__ inline ScoreCtx make_score_ctx(const FaScoreSpec& s, float scale, int h, int Tkv) {
  ScoreCtx c;
  c.flags = s.flags;
  c.scale = scale;
  c.k_log2 = scale * kLog2e;
  c.slope = (s.flags & FA_SCORE_ALIBI) ? s.alibi_slopes[h] : 0.f;
  c.slope_log2 = c.slope * kLog2e;
  c.cap = (s.flags & FA_SCORE_SOFTCAP) ? s.softcap : 1.f;
  c.cap_log2 = c.cap * kLog2e;
  c.inv_cap = 1.f / c.cap;
  c.bias = (s.flags & FA_SCORE_REL_BIAS) ? s.rel_bias + (int64_t)h * s.rel_bias_stride_h : nullptr;
  c.bias_off = s.rel_bias_center > 0 ? s.rel_bias_center : Tkv - 1;
  return c;
}

__device__ __forceinline__ float fast_tanh(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Modified logit in the log2 domain, from the raw dot product q.k.
template <int SK>
__device__ __forceinline__ float score_log2(float qk, int q, int kv, const ScoreCtx& c) {
  if constexpr (SK == SC_NONE) {
    return qk * c.k_log2;
  } else if constexpr (SK == SC_ALIBI) {
    return fmaf(qk, c.k_log2, c.slope_log2 * (float)(kv - q));
  } else if constexpr (SK == SC_SOFTCAP) {
    return c.cap_log2 * fast_tanh(qk * (c.scale * c.inv_cap));
  } else {
    float s = qk * c.scale;
    if (c.flags & FA_SCORE_ALIBI) s = fmaf(c.slope, (float)(kv - q), s);
    if (c.flags & FA_SCORE_REL_BIAS) s += __ldg(c.bias + (q - kv + c.bias_off));
    if (c.flags & FA_SCORE_SOFTCAP) s = c.cap * fast_tanh(s * c.inv_cap);
    return s * kLog2e;
  }
}

// d(modified logit)/d(scaled logit); 1 unless softcap is on.  `x_log2` is the
// value score_log2 returned for the same element.
template <int SK>
__device__ __forceinline__ float score_grad(float x_log2, const ScoreCtx& c) {
  if constexpr (SK == SC_NONE || SK == SC_ALIBI) {
    return 1.f;
  } else {
    if (!(c.flags & FA_SCORE_SOFTCAP)) return 1.f;
    const float t = x_log2 / c.cap_log2;  // tanh value
    return 1.f - t * t;
  }
}

// Per-(b) mask context.  Predicates take GLOBAL positions (local + q_off / kv_off);
// Tkv holds the global end of the key range (kv_off + Tkv).
struct MaskCtx {
  int flags, left, right, Tkv;
  int q_off, kv_off;
  const int32_t* doc_q;   // row of batch b
  const int32_t* doc_kv;
  const uint8_t* table;
  int table_cols, table_block;
  const int32_t* bit_index;  // BITMASK tiles (local positions)
  const uint32_t* bits;
  int bit_rows, bit_cols;
};

__device__ inline MaskCtx make_mask_ctx(const FaMaskSpec& m, int b, int Tkv) {
  MaskCtx c;
  c.flags = m.flags;
  c.left = m.window_left;
  c.right = m.window_right;
  c.q_off = m.q_offset;
  c.kv_off = m.kv_offset;
  c.Tkv = m.kv_offset + Tkv;
  c.doc_q = (m.flags & FA_MASK_DOCUMENT) ? m.doc_q + (int64_t)b * m.doc_stride_b : nullptr;
  c.doc_kv = (m.flags & FA_MASK_DOCUMENT) ? m.doc_kv + (int64_t)b * m.doc_stride_b : nullptr;
  c.table = m.tile_table;
  c.table_cols = m.table_cols;
  c.table_block = m.table_block > 0 ? m.table_block : 1;
  c.bit_index = m.bit_index;
  c.bits = m.bits;
  c.bit_rows = m.bit_rows;
  c.bit_cols = m.bit_cols;
  return c;
}

// mask_mod(q, kv) for one element at global positions. `dq` is doc_q[q] (ignored
// without DOCUMENT).
__device__ __forceinline__ bool mask_ok(const MaskCtx& m, int q, int kv, int dq) {
  bool ok = kv < m.Tkv;
  if (m.flags & FA_MASK_CAUSAL) ok = ok && (q >= kv);
  if (m.flags & FA_MASK_WINDOW) {
    const int d = q - kv;
    if (m.left >= 0) ok = ok && (d <= m.left);
    if (m.right >= 0) ok = ok && (-d <= m.right);
  }
  if (m.flags & FA_MASK_DOCUMENT) ok = ok && (kv < m.Tkv) && (__ldg(m.doc_kv + kv) == dq);
  if (m.flags & FA_MASK_TILE_TABLE)
    ok = ok && (m.table[(q / m.table_block) * m.table_cols + kv / m.table_block] != 0);
  if ((m.flags & FA_MASK_BITMASK) && ok) {
    const int lq = q - m.q_off, lk = kv - m.kv_off;  // local positions
    if ((unsigned)(lq >> 7) >= (unsigned)m.bit_rows || (unsigned)(lk >> 7) >= (unsigned)m.bit_cols) {
      ok = false;
    } else {
      const int slot = __ldg(m.bit_index + (lq >> 7) * m.bit_cols + (lk >> 7));
      if (slot == -1) ok = false;
      else if (slot >= 0)
        ok = (__ldg(m.bits + ((int64_t)slot * 128 + (lq & 127)) * 4 + ((lk & 127) >> 5)) >> (lk & 31)) & 1u;
    }
  }
  return ok;
}

// For non-decreasing document ids: the positions [*first, *last] within [lo, hi) whose id
// equals d (an empty range gives *first > *last).  Two binary searches, log2(hi - lo)
// steps each.
__device__ inline void doc_range(const int32_t* doc, int lo, int hi, int d, int* first, int* last) {
  int a = lo, b = hi;  // first position with id >= d
  while (a < b) {
    const int m = (a + b) >> 1;
    if (__ldg(doc + m) < d) a = m + 1;
    else b = m;
  }
  int c = a, e = hi;  // first position with id > d
  while (c < e) {
    const int m = (c + e) >> 1;
    if (__ldg(doc + m) <= d) c = m + 1;
    else e = m;
  }
  *first = a;
  *last = c - 1;
}

// Row offset (in rows of nq / nkv entries) of the block tables for (b, h).
__device__ __forceinline__ int64_t table_head(const FaBlockTables& t, int b, int h) {
  const int tb = t.num_b > 1 ? b : 0;
  const int th = t.num_h > 1 ? h : 0;
  return (int64_t)tb * t.num_h + th;
}

// Launch-time arguments of the attention kernels (everything except tensor maps).
struct AttnArgs {
  int B, H, Hkv, Tq, Tkv, D;
  FaTensor q, k, v, o, dout, dq, dk, dv;
  float* lse;
  const float* lse_in;  // [B*H, Tq] natural-log logsumexp from the forward pass
  int Tq_pad;           // Tq rounded up to 128: row length of lse2 and delta
  float* lse2;          // [B*H, Tq_pad] lse * log2(e); +inf on padding and empty rows
  float* delta;         // [B*H, Tq_pad] rowsum(O * dO); 0 on padding
  float* dq_accum;      // [B*H, Tq, D] fp32 dQ accumulator (unscaled); room for B*H*Tq_pad*D
  float scale;
  FaMaskSpec mask;
  FaScoreSpec score;
  FaBlockTables bt;
  int num_stages;
  int* status;
};

// Heads per grid group (see grid_unit_head); 0 = one group of all heads.
#ifndef FA_HEAD_GROUP
#define FA_HEAD_GROUP 8
#endif

// CTA -> (work unit, head) with the heads in groups of FA_HEAD_GROUP: the grid walks group by
// group, and inside a group unit-major (unit 0 of every head of the group, then unit 1, ...),
// so the CTAs resident at one time share a few heads' K/V, Q, dO and dQ rows in L2 instead
// of spreading over every head, while the heaviest units of each group still start first.
__device__ __forceinline__ void grid_unit_head(int x, int nunits, int nheads, int* unit, int* head) {
  const int hg = (FA_HEAD_GROUP > 0 && FA_HEAD_GROUP < nheads) ? FA_HEAD_GROUP : nheads;
  const int g = x / (hg * nunits), in = x - g * hg * nunits;
  const int cnt = min(hg, nheads - g * hg);  // heads in this group (the last may be short)
  *unit = in / cnt;
  *head = g * hg + in % cnt;
}

__device__ __forceinline__ void report_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

}  // namespace fa
