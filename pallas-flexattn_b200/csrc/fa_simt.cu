// Generic CUDA-core FlexAttention kernels: fp32 or bf16 inputs, any head dim that
// is a multiple of 8 up to 256, any block-table tile size, ragged sequence ends.
//
// They serve the shapes the tcgen05 kernels do not take (fp32 — the reference's
// CPU-sized configuration — and odd head dims or block sizes).  Math follows the
// reference kernels (src/pallas_flexattn/flash_attn.py): the forward is the online
// softmax recurrence of flash_attention_fwd_kernel (:76-106), the backward is the
// dQ kernel (:313-356) and the dK/dV kernel (:206-253), here restricted to the
// tiles the block tables list.  Exact expf/tanhf are used so fp32 results track
// the fp32 reference closely.
//
// Layout: a CTA of 8 warps takes 8 consecutive rows of one block-table row (the
// rows share a tile list); K/V (or Q/dO) arrive in 32-row chunks staged in shared
// memory with a padded stride so lane j reading row j is bank-conflict free.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "fa_common.cuh"
#include "fa_internal.h"

namespace fa {
namespace {

constexpr int kWarps = 8;
constexpr int kChunk = 32;
constexpr int kMaxDPerLane = 8;  // D <= 256

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// score_mod in natural units with exact math; returns the modified logit and
// (through *grad) its derivative w.r.t. the scaled logit.
__device__ __forceinline__ float score_nat(float qk, int q, int kv, const ScoreCtx& c, float* grad) {
  float s = qk * c.scale;
  if (c.flags & FA_SCORE_ALIBI) s += c.slope * (float)(kv - q);
  if (c.flags & FA_SCORE_REL_BIAS) s += c.bias[q - kv + c.bias_off];
  float g = 1.f;
  if (c.flags & FA_SCORE_SOFTCAP) {
    const float t = tanhf(s * c.inv_cap);
    s = c.cap * t;
    g = 1.f - t * t;
  }
  if (grad) *grad = g;
  return s;
}

template <typename T>
__device__ __forceinline__ const T* row_ptr(const FaTensor& t, int b, int h, int r) {
  return reinterpret_cast<const T*>(t.ptr) + (int64_t)b * t.stride_b + (int64_t)h * t.stride_h +
         (int64_t)r * t.stride_t;
}
template <typename T>
__device__ __forceinline__ T* row_ptr_w(const FaTensor& t, int b, int h, int r) {
  return reinterpret_cast<T*>(t.ptr) + (int64_t)b * t.stride_b + (int64_t)h * t.stride_h + (int64_t)r * t.stride_t;
}

// Entry e of the merged (partial, then full) list of a table row.
struct RowList {
  const int32_t* part;
  const int32_t* full;
  int n_part, n_full;
  __device__ int count() const { return n_part + n_full; }
  __device__ int at(int e, bool* partial) const {
    *partial = e < n_part;
    return e < n_part ? part[e] : full[e - n_part];
  }
};

__device__ RowList row_list(const int32_t* num, const int32_t* idx, const int32_t* fnum, const int32_t* fidx,
                            int64_t row, int cap) {
  RowList r;
  r.n_part = num ? num[row] : 0;
  r.n_full = fnum ? fnum[row] : 0;
  r.part = idx ? idx + row * cap : nullptr;
  r.full = fidx ? fidx + row * cap : nullptr;
  return r;
}

// ------------------------------------------------------------------------ forward
template <typename T>
__global__ void __launch_bounds__(kWarps * 32) fwd_simt_kernel(const AttnArgs a) {
  extern __shared__ float sm[];
  const int D = a.D, DP = D + 1;
  float* sK = sm;                  // [kChunk][DP]
  float* sV = sK + kChunk * DP;    // [kChunk][DP]
  float* sQ = sV + kChunk * DP;    // [kWarps][D]

  const int bq = a.bt.block_q, bkv = a.bt.block_kv;
  const int groups = (bq + kWarps - 1) / kWarps;
  const int qb = blockIdx.x / groups, grp = blockIdx.x % groups;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H, hk = h / (a.H / a.Hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int in_blk = grp * kWarps + warp;
  const int q_row = qb * bq + in_blk;
  const bool row_ok = in_blk < bq && q_row < a.Tq;

  const ScoreCtx sc = make_score_ctx(a.score, a.scale, h, a.Tkv);
  const MaskCtx mc = make_mask_ctx(a.mask, b, a.Tkv);
  const int dq_val = (mc.flags & FA_MASK_DOCUMENT) && row_ok ? mc.doc_q[q_row + mc.q_off] : 0;

  if (row_ok) {
    const T* q = row_ptr<T>(a.q, b, h, q_row);
    for (int d = lane; d < D; d += 32) sQ[warp * D + d] = to_f(q[d]);
  }
  const int64_t trow = table_head(a.bt, b, h) * a.bt.nq + qb;
  const RowList L = row_list(a.bt.kv_num_blocks, a.bt.kv_indices, a.bt.full_kv_num_blocks, a.bt.full_kv_indices, trow,
                             a.bt.kv_cap);
  float m = -INFINITY, l = 0.f, o[kMaxDPerLane];
#pragma unroll
  for (int u = 0; u < kMaxDPerLane; ++u) o[u] = 0.f;

  for (int e = 0; e < L.count(); ++e) {
    bool partial;
    const int j = L.at(e, &partial);
    if (j < 0 || j >= a.bt.nkv) continue;
    const int t_end = min((j + 1) * bkv, a.Tkv);
    for (int c0 = j * bkv; c0 < t_end; c0 += kChunk) {
      __syncthreads();
      for (int idx = threadIdx.x; idx < kChunk * D; idx += blockDim.x) {
        const int r = idx / D, d = idx % D, kv = c0 + r;
        float kx = 0.f, vx = 0.f;
        if (kv < t_end) {
          kx = to_f(row_ptr<T>(a.k, b, hk, kv)[d]);
          vx = to_f(row_ptr<T>(a.v, b, hk, kv)[d]);
        }
        sK[r * DP + d] = kx;
        sV[r * DP + d] = vx;
      }
      __syncthreads();
      if (!row_ok) continue;
      const int kv = c0 + lane;
      float dot = 0.f;
      for (int d = 0; d < D; ++d) dot = fmaf(sQ[warp * D + d], sK[lane * DP + d], dot);
      float x = score_nat(dot, q_row + mc.q_off, kv + mc.kv_off, sc, nullptr);
      if (kv >= t_end || (partial && !mask_ok(mc, q_row + mc.q_off, kv + mc.kv_off, dq_val))) x = -INFINITY;
      const float m_new = fmaxf(m, warp_max(x));
      const float alpha = (m_new == -INFINITY) ? 1.f : expf(m - m_new);
      const float p = (m_new == -INFINITY) ? 0.f : expf(x - m_new);
      l = l * alpha + warp_sum(p);
#pragma unroll
      for (int u = 0; u < kMaxDPerLane; ++u) o[u] *= alpha;
      for (int jj = 0; jj < kChunk; ++jj) {
        const float pj = __shfl_sync(0xffffffffu, p, jj);
        if (pj == 0.f) continue;
#pragma unroll
        for (int u = 0; u < kMaxDPerLane; ++u) {
          const int d = lane + 32 * u;
          if (d < D) o[u] = fmaf(pj, sV[jj * DP + d], o[u]);
        }
      }
      m = m_new;
    }
  }
  if (!row_ok) return;
  const bool live = l > 0.f;
  const float inv = live ? 1.f / l : 0.f;
  T* orow = row_ptr_w<T>(a.o, b, h, q_row);
#pragma unroll
  for (int u = 0; u < kMaxDPerLane; ++u) {
    const int d = lane + 32 * u;
    if (d < D) orow[d] = from_f<T>(o[u] * inv);
  }
  if (lane == 0) a.lse[(int64_t)bh * a.Tq + q_row] = live ? m + logf(l) : -INFINITY;
}

// ------------------------------------------------------------------------ backward: dQ (row-wise)
// Writes the unscaled fp32 dQ row into dq_accum; the convert kernel applies `scale`.
template <typename T>
__global__ void __launch_bounds__(kWarps * 32) bwd_dq_simt_kernel(const AttnArgs a) {
  extern __shared__ float sm[];
  const int D = a.D, DP = D + 1;
  float* sK = sm;
  float* sV = sK + kChunk * DP;
  float* sQ = sV + kChunk * DP;      // [kWarps][D]
  float* sdO = sQ + kWarps * D;      // [kWarps][D]

  const int bq = a.bt.block_q, bkv = a.bt.block_kv;
  const int groups = (bq + kWarps - 1) / kWarps;
  const int qb = blockIdx.x / groups, grp = blockIdx.x % groups;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H, hk = h / (a.H / a.Hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int in_blk = grp * kWarps + warp;
  const int q_row = qb * bq + in_blk;
  const bool row_ok = in_blk < bq && q_row < a.Tq;

  const ScoreCtx sc = make_score_ctx(a.score, a.scale, h, a.Tkv);
  const MaskCtx mc = make_mask_ctx(a.mask, b, a.Tkv);
  const int dq_val = (mc.flags & FA_MASK_DOCUMENT) && row_ok ? mc.doc_q[q_row + mc.q_off] : 0;
  float lse = -INFINITY, delta = 0.f;
  if (row_ok) {
    const T* q = row_ptr<T>(a.q, b, h, q_row);
    const T* g = row_ptr<T>(a.dout, b, h, q_row);
    for (int d = lane; d < D; d += 32) {
      sQ[warp * D + d] = to_f(q[d]);
      sdO[warp * D + d] = to_f(g[d]);
    }
    lse = a.lse_in[(int64_t)bh * a.Tq + q_row];
    delta = a.delta[(int64_t)bh * a.Tq_pad + q_row];
  }
  const int64_t trow = table_head(a.bt, b, h) * a.bt.nq + qb;
  const RowList L = row_list(a.bt.kv_num_blocks, a.bt.kv_indices, a.bt.full_kv_num_blocks, a.bt.full_kv_indices, trow,
                             a.bt.kv_cap);
  float acc[kMaxDPerLane];
#pragma unroll
  for (int u = 0; u < kMaxDPerLane; ++u) acc[u] = 0.f;

  for (int e = 0; e < L.count(); ++e) {
    bool partial;
    const int j = L.at(e, &partial);
    if (j < 0 || j >= a.bt.nkv) continue;
    const int t_end = min((j + 1) * bkv, a.Tkv);
    for (int c0 = j * bkv; c0 < t_end; c0 += kChunk) {
      __syncthreads();
      for (int idx = threadIdx.x; idx < kChunk * D; idx += blockDim.x) {
        const int r = idx / D, d = idx % D, kv = c0 + r;
        float kx = 0.f, vx = 0.f;
        if (kv < t_end) {
          kx = to_f(row_ptr<T>(a.k, b, hk, kv)[d]);
          vx = to_f(row_ptr<T>(a.v, b, hk, kv)[d]);
        }
        sK[r * DP + d] = kx;
        sV[r * DP + d] = vx;
      }
      __syncthreads();
      if (!row_ok) continue;
      const int kv = c0 + lane;
      float dot = 0.f, dp = 0.f;
      for (int d = 0; d < D; ++d) {
        dot = fmaf(sQ[warp * D + d], sK[lane * DP + d], dot);
        dp = fmaf(sdO[warp * D + d], sV[lane * DP + d], dp);
      }
      float g;
      const float x = score_nat(dot, q_row + mc.q_off, kv + mc.kv_off, sc, &g);
      const bool live = kv < t_end && !(partial && !mask_ok(mc, q_row + mc.q_off, kv + mc.kv_off, dq_val)) && lse != -INFINITY;
      const float p = live ? expf(x - lse) : 0.f;
      const float ds = p * (dp - delta) * g;
      for (int jj = 0; jj < kChunk; ++jj) {
        const float dj = __shfl_sync(0xffffffffu, ds, jj);
        if (dj == 0.f) continue;
#pragma unroll
        for (int u = 0; u < kMaxDPerLane; ++u) {
          const int d = lane + 32 * u;
          if (d < D) acc[u] = fmaf(dj, sK[jj * DP + d], acc[u]);
        }
      }
    }
  }
  if (!row_ok) return;
  float* out = a.dq_accum + ((int64_t)bh * a.Tq + q_row) * D;
#pragma unroll
  for (int u = 0; u < kMaxDPerLane; ++u) {
    const int d = lane + 32 * u;
    if (d < D) out[d] = acc[u];
  }
}

// ------------------------------------------------------------------------ backward: dK, dV (column-wise)
template <typename T>
__global__ void __launch_bounds__(kWarps * 32) bwd_dkv_simt_kernel(const AttnArgs a) {
  extern __shared__ float sm[];
  const int D = a.D, DP = D + 1;
  float* sQ = sm;                    // [kChunk][DP]
  float* sdO = sQ + kChunk * DP;     // [kChunk][DP]
  float* sK = sdO + kChunk * DP;     // [kWarps][D]
  float* sV = sK + kWarps * D;       // [kWarps][D]
  float* sL = sV + kWarps * D;       // [kChunk] lse
  float* sDl = sL + kChunk;          // [kChunk] delta
  int* sDoc = reinterpret_cast<int*>(sDl + kChunk);  // [kChunk] doc ids of the staged q rows

  const int bq = a.bt.block_q, bkv = a.bt.block_kv;
  const int groups = (bkv + kWarps - 1) / kWarps;
  const int kb = blockIdx.x / groups, grp = blockIdx.x % groups;
  // One block per (kv block, b, kv head); dK and dV sum over the G = H / Hkv query heads of
  // the group (grouped-query attention; G = 1 otherwise).
  const int G = a.H / a.Hkv;
  const int bhk = blockIdx.y, b = bhk / a.Hkv, hk = bhk % a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int in_blk = grp * kWarps + warp;
  const int kv_row = kb * bkv + in_blk;
  const bool row_ok = in_blk < bkv && kv_row < a.Tkv;

  const MaskCtx mc = make_mask_ctx(a.mask, b, a.Tkv);
  if (row_ok) {
    const T* k = row_ptr<T>(a.k, b, hk, kv_row);
    const T* v = row_ptr<T>(a.v, b, hk, kv_row);
    for (int d = lane; d < D; d += 32) {
      sK[warp * D + d] = to_f(k[d]);
      sV[warp * D + d] = to_f(v[d]);
    }
  }
  float dk[kMaxDPerLane], dv[kMaxDPerLane];
#pragma unroll
  for (int u = 0; u < kMaxDPerLane; ++u) dk[u] = dv[u] = 0.f;

  for (int gi = 0; gi < G; ++gi) {
  const int h = hk * G + gi, bh = b * a.H + h;
  const ScoreCtx sc = make_score_ctx(a.score, a.scale, h, a.Tkv);
  const int64_t tcol = table_head(a.bt, b, h) * a.bt.nkv + kb;
  const RowList L =
      row_list(a.bt.q_num_blocks, a.bt.q_indices, a.bt.full_q_num_blocks, a.bt.full_q_indices, tcol, a.bt.q_cap);
  for (int e = 0; e < L.count(); ++e) {
    bool partial;
    const int i = L.at(e, &partial);
    if (i < 0 || i >= a.bt.nq) continue;
    const int t_end = min((i + 1) * bq, a.Tq);
    for (int c0 = i * bq; c0 < t_end; c0 += kChunk) {
      __syncthreads();
      for (int idx = threadIdx.x; idx < kChunk * D; idx += blockDim.x) {
        const int r = idx / D, d = idx % D, q = c0 + r;
        float qx = 0.f, gx = 0.f;
        if (q < t_end) {
          qx = to_f(row_ptr<T>(a.q, b, h, q)[d]);
          gx = to_f(row_ptr<T>(a.dout, b, h, q)[d]);
        }
        sQ[r * DP + d] = qx;
        sdO[r * DP + d] = gx;
      }
      for (int r = threadIdx.x; r < kChunk; r += blockDim.x) {
        const int q = c0 + r;
        sL[r] = q < t_end ? a.lse_in[(int64_t)bh * a.Tq + q] : -INFINITY;
        sDl[r] = q < t_end ? a.delta[(int64_t)bh * a.Tq_pad + q] : 0.f;
        sDoc[r] = (q < t_end && (mc.flags & FA_MASK_DOCUMENT)) ? mc.doc_q[q + mc.q_off] : 0;
      }
      __syncthreads();
      if (!row_ok) continue;
      const int q = c0 + lane;
      float dot = 0.f, dp = 0.f;
      for (int d = 0; d < D; ++d) {
        dot = fmaf(sQ[lane * DP + d], sK[warp * D + d], dot);
        dp = fmaf(sdO[lane * DP + d], sV[warp * D + d], dp);
      }
      float g;
      const float x = score_nat(dot, q + mc.q_off, kv_row + mc.kv_off, sc, &g);
      const float lse = sL[lane];
      const bool live = q < t_end && !(partial && !mask_ok(mc, q + mc.q_off, kv_row + mc.kv_off, sDoc[lane])) && lse != -INFINITY;
      const float p = live ? expf(x - lse) : 0.f;
      const float ds = p * (dp - sDl[lane]) * g;
      for (int jj = 0; jj < kChunk; ++jj) {
        const float pj = __shfl_sync(0xffffffffu, p, jj);
        const float dj = __shfl_sync(0xffffffffu, ds, jj);
        if (pj == 0.f && dj == 0.f) continue;
#pragma unroll
        for (int u = 0; u < kMaxDPerLane; ++u) {
          const int d = lane + 32 * u;
          if (d < D) {
            dv[u] = fmaf(pj, sdO[jj * DP + d], dv[u]);
            dk[u] = fmaf(dj, sQ[jj * DP + d], dk[u]);
          }
        }
      }
    }
  }
  }  // heads of the group
  if (!row_ok) return;
  T* dkr = row_ptr_w<T>(a.dk, b, hk, kv_row);
  T* dvr = row_ptr_w<T>(a.dv, b, hk, kv_row);
#pragma unroll
  for (int u = 0; u < kMaxDPerLane; ++u) {
    const int d = lane + 32 * u;
    if (d < D) {
      dkr[d] = from_f<T>(dk[u] * a.scale);
      dvr[d] = from_f<T>(dv[u]);
    }
  }
}

template <typename K>
cudaError_t launch_simt(K kern, dim3 grid, size_t smem, cudaStream_t stream, const AttnArgs& a) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kWarps * 32, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_fwd_simt(const AttnArgs& a, int dtype, cudaStream_t stream) {
  const int groups = (a.bt.block_q + kWarps - 1) / kWarps;
  const dim3 grid((unsigned)(a.bt.nq * groups), (unsigned)(a.B * a.H));
  const size_t smem = (size_t)(2 * kChunk * (a.D + 1) + kWarps * a.D) * sizeof(float);
  if (dtype == FA_DTYPE_F32) return launch_simt(fwd_simt_kernel<float>, grid, smem, stream, a);
  return launch_simt(fwd_simt_kernel<__nv_bfloat16>, grid, smem, stream, a);
}

cudaError_t launch_bwd_simt(const AttnArgs& a, int dtype, cudaStream_t stream) {
  {
    const int groups = (a.bt.block_q + kWarps - 1) / kWarps;
    const dim3 grid((unsigned)(a.bt.nq * groups), (unsigned)(a.B * a.H));
    const size_t smem = (size_t)(2 * kChunk * (a.D + 1) + 2 * kWarps * a.D) * sizeof(float);
    cudaError_t e = dtype == FA_DTYPE_F32 ? launch_simt(bwd_dq_simt_kernel<float>, grid, smem, stream, a)
                                          : launch_simt(bwd_dq_simt_kernel<__nv_bfloat16>, grid, smem, stream, a);
    if (e != cudaSuccess) return e;
  }
  const int groups = (a.bt.block_kv + kWarps - 1) / kWarps;
  const dim3 grid((unsigned)(a.bt.nkv * groups), (unsigned)(a.B * a.Hkv));
  const size_t smem = (size_t)(2 * kChunk * (a.D + 1) + 2 * kWarps * a.D + 3 * kChunk) * sizeof(float);
  return dtype == FA_DTYPE_F32 ? launch_simt(bwd_dkv_simt_kernel<float>, grid, smem, stream, a)
                               : launch_simt(bwd_dkv_simt_kernel<__nv_bfloat16>, grid, smem, stream, a);
}

}  // namespace fa
