// Split-KV decode: a few new query tokens per sequence against a K/V cache (fa_decode).
//
// Decode reads the whole cache once per call and does O(G * Tq) multiply-adds per cache
// element, so with a handful of query rows it is bound by HBM bandwidth.  The cache of each
// (b, K/V head) is cut into num_splits chunks; one CTA per (chunk, b, K/V head) handles
// every query row of the K/V head's group (G = H / H_kv heads x Tq tokens = M rows,
// M <= 64), so each cache element is read from HBM once for all of them.
//
// Per CTA: TMA streams 64-row K and V tiles (128-byte swizzled panels) through a ring of
// stages guarded by mbarriers; the 256 threads then run, per tile,
//   scores   thread = (cache row j, every 4th query row): 16-byte K chunks against fp32 Q
//            (the swizzle spreads the 32 rows a warp reads over all banks),
//   softmax  warp = query row, online (running max and sum per row),
//   P V      thread = (8 output columns, every RG-th query row), fp32 accumulators in
//            registers, probabilities read 4 cache rows at a time,
// and thread 0 refills the stage.  Each CTA writes its normalised partial (o, lse) to the
// workspace; decode_merge_kernel combines the chunks by log-sum-exp.  Query row i of batch b
// sits at global position kv_lens[b] - Tq + i.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdio>

#include "fa_common.cuh"
#include "fa_internal.h"
#include "fa_ptx.cuh"
#include "flexattn.h"

namespace fa {
namespace {

constexpr int kDecThreads = 256;
constexpr int kDecKT = 64;          // cache rows per tile (the TMA box height)
constexpr int kDecMaxRows = 64;     // G * Tq
constexpr int kDecPS = kDecKT + 4;  // row stride of the score tile in floats (16-byte aligned, bank-shifted)
constexpr int kPanelBytes = kDecKT * 128;

struct DecodeArgs {
  int B, H, Hkv, Tq, Tkv, D, G, M, splits, chunk, stages;
  FaTensor q, o;
  float* lse;
  const int32_t* kv_lens;
  float scale;
  FaMaskSpec mask;
  FaScoreSpec score;
  float* part_o;    // [splits, B*H*Tq, D]
  float* part_lse;  // [splits, B*H*Tq]
  int* status;
};

// Dynamic shared memory of one CTA (bytes), including 1024 bytes of alignment slack.
inline size_t decode_smem_bytes(int D, int es, int M, int stages) {
  const int Mp = (M + 3) & ~3;
  return 1024 + (size_t)stages * 2 * kDecKT * D * es + (size_t)Mp * D * 4 + (size_t)Mp * kDecPS * 4 +
         4 * kDecMaxRows * 4 + (size_t)stages * 8 + 16;
}

__device__ __forceinline__ float dec_ld(const float* p) { return *p; }
__device__ __forceinline__ float dec_ld(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// Element values of one 16-byte chunk.
__device__ __forceinline__ void unpack_chunk(const uint4 raw, float (&f)[4]) {
  f[0] = __uint_as_float(raw.x);
  f[1] = __uint_as_float(raw.y);
  f[2] = __uint_as_float(raw.z);
  f[3] = __uint_as_float(raw.w);
}
__device__ __forceinline__ void unpack_chunk(const uint4 raw, float (&f)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// Byte offset of 16-byte chunk c (counted along the row) of row r in a tile of 128-byte
// swizzled panels: panel c / 8, chunk slot (c % 8) ^ (r % 8) of the row's 128-byte line.
__device__ __forceinline__ uint32_t chunk_off(int r, int c) {
  return (uint32_t)((c >> 3) * kPanelBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

template <typename T, int D>
__global__ void __launch_bounds__(kDecThreads, D <= 128 ? 2 : 1)
    decode_split_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                        const DecodeArgs a) {
  constexpr int ES = (int)sizeof(T);
  constexpr int EPC = 16 / ES;           // elements per 16-byte chunk
  constexpr int CHUNKS = D / EPC;        // chunks per row
  constexpr int NPANEL = D * ES / 128;   // 128-byte panels per row
  constexpr int TILE = kDecKT * D * ES;  // bytes of one K (or V) tile
  constexpr int NCG = D / 8;             // P V phase: groups of 8 output columns
  constexpr int RG = kDecThreads / NCG;  //            query-row groups
  constexpr int RPT = kDecMaxRows / RG;  //            rows per thread, at most
  constexpr int SPT = kDecMaxRows / 4;   // score phase: rows per thread, at most

  extern __shared__ unsigned char dsm_raw[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages, M = a.M, Mp = (M + 3) & ~3;
  float* sQ = reinterpret_cast<float*>(base + (size_t)S * 2 * TILE);  // [Mp][D], pre-scaled
  float* sP = sQ + Mp * D;                                             // [Mp][kDecPS]
  float* sMax = sP + Mp * kDecPS;  // running max per row (log2 domain)
  float* sSum = sMax + kDecMaxRows;
  float* sAlpha = sSum + kDecMaxRows;
  float* sSlope = sAlpha + kDecMaxRows;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSlope + kDecMaxRows);
  volatile int* never = reinterpret_cast<volatile int*>(bars + S);  // stays 0: waits end by time only

  const int s = blockIdx.x, bhk = blockIdx.y, b = bhk / a.Hkv, hk = bhk % a.Hkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int len = a.kv_lens ? min(max(__ldg(a.kv_lens + b), 0), a.Tkv) : a.Tkv;
  const int kv0 = s * a.chunk, kv1 = min(kv0 + a.chunk, len);
  const int ntiles = kv1 > kv0 ? (kv1 - kv0 + kDecKT - 1) / kDecKT : 0;
  const int qbase = len - a.Tq;  // global position of query token 0

  auto issue = [&](int t) {  // thread 0 only
    const int st = t % S;
    unsigned char* dst = base + (size_t)st * 2 * TILE;
    mbar_arrive_expect_tx(bars + st, 2 * TILE);
#pragma unroll
    for (int p = 0; p < NPANEL; ++p) {
      tma_load_4d(dst + p * kPanelBytes, &tk, bars + st, p * (128 / ES), kv0 + t * kDecKT, hk, b);
      tma_load_4d(dst + TILE + p * kPanelBytes, &tv, bars + st, p * (128 / ES), kv0 + t * kDecKT, hk, b);
    }
  };
  if (tid == 0) {
    for (int i = 0; i < S; ++i) mbar_init(bars + i, 1);
    *never = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    for (int t = 0; t < min(S, ntiles); ++t) issue(t);
  }
  for (int e = tid; e < M * D; e += kDecThreads) {
    const int m = e / D, d = e % D, g = m / a.Tq, i = m % a.Tq;
    const T* qp = reinterpret_cast<const T*>(a.q.ptr) + (int64_t)b * a.q.stride_b +
                  (int64_t)(hk * a.G + g) * a.q.stride_h + (int64_t)i * a.q.stride_t;
    sQ[e] = dec_ld(qp + d) * a.scale;
  }
  for (int m = tid; m < kDecMaxRows; m += kDecThreads) {
    sMax[m] = -INFINITY;
    sSum[m] = 0.f;
    sAlpha[m] = 1.f;
    sSlope[m] = (m < M && (a.score.flags & FA_SCORE_ALIBI)) ? a.score.alibi_slopes[hk * a.G + m / a.Tq] : 0.f;
  }
  const bool softcap = (a.score.flags & FA_SCORE_SOFTCAP) != 0;
  const float cap = softcap ? a.score.softcap : 1.f, inv_cap = 1.f / cap;
  const int mflags = a.mask.flags, left = a.mask.window_left, right = a.mask.window_right;

  const int cg = tid % NCG, rg = tid / NCG;          // P V phase
  const int jrow = tid % kDecKT, mg = tid / kDecKT;  // score phase
  float acc[RPT][8];
#pragma unroll
  for (int r = 0; r < RPT; ++r)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[r][e] = 0.f;

  int it = 0;
  bool ok = true;
  for (; it < ntiles; ++it) {
    const int st = it % S, t0 = kv0 + it * kDecKT, n = min(kDecKT, kv1 - t0);
    const unsigned char* kst = base + (size_t)st * 2 * TILE;
    unsigned char* vst = base + (size_t)st * 2 * TILE + TILE;
    const bool got = mbar_wait(bars + st, (uint32_t)((it / S) & 1), never);
    if (__syncthreads_or(!got)) {
      ok = false;
      break;
    }
    if (n < kDecKT) {  // rows past the chunk's end hold other data: zero them in V
      for (int e = tid; e < (kDecKT - n) * CHUNKS; e += kDecThreads)
        *reinterpret_cast<uint4*>(vst + chunk_off(n + e / CHUNKS, e % CHUNKS)) = make_uint4(0, 0, 0, 0);
      __syncthreads();
    }

    // ---- scores (log2 domain), masked to -inf
    {
      float dot[SPT];
#pragma unroll
      for (int r = 0; r < SPT; ++r) dot[r] = 0.f;
#pragma unroll 2
      for (int c = 0; c < CHUNKS; ++c) {
        float kf[EPC];
        unpack_chunk(*reinterpret_cast<const uint4*>(kst + chunk_off(jrow, c)), kf);
#pragma unroll
        for (int r = 0; r < SPT; ++r) {
          const int m = mg + 4 * r;
          if (m < M) {
            const float4* q4 = reinterpret_cast<const float4*>(sQ + m * D + c * EPC);
#pragma unroll
            for (int e4 = 0; e4 < EPC / 4; ++e4) {
              const float4 qx = q4[e4];
              dot[r] = fmaf(kf[4 * e4], qx.x, dot[r]);
              dot[r] = fmaf(kf[4 * e4 + 1], qx.y, dot[r]);
              dot[r] = fmaf(kf[4 * e4 + 2], qx.z, dot[r]);
              dot[r] = fmaf(kf[4 * e4 + 3], qx.w, dot[r]);
            }
          }
        }
      }
      const int kvpos = t0 + jrow;
#pragma unroll
      for (int r = 0; r < SPT; ++r) {
        const int m = mg + 4 * r;
        if (m >= M) continue;
        const int qpos = qbase + m % a.Tq;
        float x = fmaf(sSlope[m], (float)(kvpos - qpos), dot[r]);
        if (softcap) x = cap * fast_tanh(x * inv_cap);
        bool keep = jrow < n;
        if (mflags & FA_MASK_CAUSAL) keep = keep && kvpos <= qpos;
        if (mflags & FA_MASK_WINDOW) {
          if (left >= 0) keep = keep && qpos - kvpos <= left;
          if (right >= 0) keep = keep && kvpos - qpos <= right;
        }
        sP[m * kDecPS + jrow] = keep ? x * kLog2e : -INFINITY;
      }
    }
    __syncthreads();
    // ---- online softmax, one warp per row
    for (int m = warp; m < M; m += kDecThreads / 32) {
      const float x0 = sP[m * kDecPS + lane], x1 = sP[m * kDecPS + lane + 32];
      float mx = fmaxf(x0, x1);
#pragma unroll
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mold = sMax[m], mnew = fmaxf(mold, mx);
      const float p0 = mnew == -INFINITY ? 0.f : exp2f(x0 - mnew);
      const float p1 = mnew == -INFINITY ? 0.f : exp2f(x1 - mnew);
      float sum = p0 + p1;
#pragma unroll
      for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      sP[m * kDecPS + lane] = p0;
      sP[m * kDecPS + lane + 32] = p1;
      if (lane == 0) {
        const float alpha = mold == -INFINITY ? 0.f : exp2f(mold - mnew);
        sAlpha[m] = alpha;
        sSum[m] = sSum[m] * alpha + sum;
        sMax[m] = mnew;
      }
    }
    __syncthreads();
    // ---- P V over the tile's first n rows, rounded up to 4 (the rows past n are zero)
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
      const int m = rg + RG * r;
      if (m < M) {
        const float al = sAlpha[m];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[r][e] *= al;
      }
    }
    for (int j0 = 0; j0 < n; j0 += 4) {
      float4 p4[RPT];
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const int m = rg + RG * r;
        p4[r] = m < M ? *reinterpret_cast<const float4*>(sP + m * kDecPS + j0) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int j = j0 + jj;
        float vf[8];
        if constexpr (ES == 2) {
          unpack_chunk(*reinterpret_cast<const uint4*>(vst + chunk_off(j, cg)), vf);
        } else {
          float lo[4], hi[4];
          unpack_chunk(*reinterpret_cast<const uint4*>(vst + chunk_off(j, 2 * cg)), lo);
          unpack_chunk(*reinterpret_cast<const uint4*>(vst + chunk_off(j, 2 * cg + 1)), hi);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            vf[e] = lo[e];
            vf[4 + e] = hi[e];
          }
        }
#pragma unroll
        for (int r = 0; r < RPT; ++r) {
          const float pj = jj == 0 ? p4[r].x : jj == 1 ? p4[r].y : jj == 2 ? p4[r].z : p4[r].w;
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[r][e] = fmaf(pj, vf[e], acc[r][e]);
        }
      }
    }
    __syncthreads();
    if (tid == 0 && it + S < ntiles) {
      fence_proxy_async_smem();
      issue(it + S);
    }
  }
  if (!ok) {
    if (tid == 0) {
      report_status(a.status, FA_ERR_TIMEOUT);
      // tiles still in flight land in this CTA's shared memory: let them finish (bounded)
      for (int t = it; t < min(it + S, ntiles); ++t) mbar_wait(bars + t % S, (uint32_t)((t / S) & 1), never);
    }
    __syncthreads();
    return;
  }
  // ---- this chunk's normalised partial (o, lse); an empty chunk gives o = 0, lse = -inf
  const int64_t rows = (int64_t)a.B * a.H * a.Tq;
#pragma unroll
  for (int r = 0; r < RPT; ++r) {
    const int m = rg + RG * r;
    if (m >= M) continue;
    const int g = m / a.Tq, i = m % a.Tq;
    const int64_t row = ((int64_t)b * a.H + hk * a.G + g) * a.Tq + i;
    const float l = sSum[m], inv = l > 0.f ? 1.f / l : 0.f;
    float4* dst = reinterpret_cast<float4*>(a.part_o + ((int64_t)s * rows + row) * D + cg * 8);
    dst[0] = make_float4(acc[r][0] * inv, acc[r][1] * inv, acc[r][2] * inv, acc[r][3] * inv);
    dst[1] = make_float4(acc[r][4] * inv, acc[r][5] * inv, acc[r][6] * inv, acc[r][7] * inv);
    if (cg == 0) a.part_lse[(int64_t)s * rows + row] = l > 0.f ? (sMax[m] + log2f(l)) * kLn2 : -INFINITY;
  }
}

// One warp per output row: log-sum-exp merge of the chunks' partials into o and lse.
template <typename T>
__global__ void __launch_bounds__(256) decode_merge_kernel(const DecodeArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)a.B * a.H * a.Tq;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (row >= rows) return;
  float L = -INFINITY;
  for (int s = 0; s < a.splits; ++s) L = fmaxf(L, a.part_lse[(int64_t)s * rows + row]);
  float wsum = 0.f;
  for (int s = 0; s < a.splits; ++s) {
    const float ls = a.part_lse[(int64_t)s * rows + row];
    wsum += ls == -INFINITY ? 0.f : expf(ls - L);
  }
  const int i = (int)(row % a.Tq), bh = (int)(row / a.Tq), b = bh / a.H, h = bh % a.H;
  T* o = reinterpret_cast<T*>(a.o.ptr) + (int64_t)b * a.o.stride_b + (int64_t)h * a.o.stride_h +
         (int64_t)i * a.o.stride_t;
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  for (int d = lane; d < a.D; d += 32) {
    float acc = 0.f;
    for (int s = 0; s < a.splits; ++s) {
      const float ls = a.part_lse[(int64_t)s * rows + row];
      if (ls != -INFINITY) acc = fmaf(expf(ls - L), a.part_o[((int64_t)s * rows + row) * a.D + d], acc);
    }
    if constexpr (sizeof(T) == 4) o[d] = acc * inv;
    else o[d] = __float2bfloat16_rn(acc * inv);
  }
  if (lane == 0) a.lse[row] = wsum > 0.f ? L + logf(wsum) : -INFINITY;
}

// Chunking and pipeline depth for a call.
struct DecodePlan {
  int splits, chunk, stages;
  size_t smem;
};

DecodePlan plan_decode(const FaDecodeParams* p) {
  DecodePlan pl;
  const int es = p->dtype == FA_DTYPE_F32 ? 4 : 2;
  const int M = (p->H / p->H_kv) * p->Tq;
  int sp = p->num_splits;
  if (sp <= 0) {  // about four CTAs per SM across the grid, chunks of at least 256 cache rows
    const int ctas = p->B * p->H_kv;
    sp = (4 * 148 + ctas - 1) / ctas;
    const int max_sp = (p->Tkv + 255) / 256;
    if (sp > max_sp) sp = max_sp;
    if (sp < 1) sp = 1;
  }
  if (sp > p->Tkv) sp = p->Tkv;
  int ch = (p->Tkv + sp - 1) / sp;
  ch = (ch + kDecKT - 1) / kDecKT * kDecKT;  // chunks start on tile boundaries
  pl.chunk = ch;
  pl.splits = (p->Tkv + ch - 1) / ch;
  // stages: as many (<= 4) as leave room for two CTAs per SM; else two, else one
  const size_t fixed = decode_smem_bytes(p->D, es, M, 0), stage = decode_smem_bytes(p->D, es, M, 1) - fixed;
  const size_t two_ctas = 113 * 1024, one_cta = 220 * 1024;
  int S = fixed + stage <= two_ctas ? (int)((two_ctas - fixed) / stage) : (fixed + 2 * stage <= one_cta ? 2 : 1);
  if (S > 4) S = 4;
  pl.stages = S;
  pl.smem = decode_smem_bytes(p->D, es, M, S);
  return pl;
}

int check_decode(const FaDecodeParams* p) {
  char msg[192];
  if (!p) return set_last_error(FA_ERR_INVALID, "fa_decode: params is NULL");
  if (p->dtype != FA_DTYPE_BF16 && p->dtype != FA_DTYPE_F32)
    return set_last_error(FA_ERR_INVALID, "fa_decode: unknown dtype");
  if (p->B <= 0 || p->H <= 0 || p->H_kv <= 0 || p->Tq <= 0 || p->Tkv <= 0 || p->D <= 0) {
    snprintf(msg, sizeof(msg), "fa_decode: non-positive shape B=%d H=%d H_kv=%d Tq=%d Tkv=%d D=%d", p->B, p->H,
             p->H_kv, p->Tq, p->Tkv, p->D);
    return set_last_error(FA_ERR_INVALID, msg);
  }
  if (p->H % p->H_kv) return set_last_error(FA_ERR_INVALID, "fa_decode: H must be a multiple of H_kv");
  if (p->D != 64 && p->D != 128 && p->D != 256) {
    snprintf(msg, sizeof(msg), "fa_decode: head dim %d (supported: 64, 128, 256)", p->D);
    return set_last_error(FA_ERR_UNSUPPORTED, msg);
  }
  if ((p->H / p->H_kv) * p->Tq > kDecMaxRows) {
    snprintf(msg, sizeof(msg), "fa_decode: H / H_kv * Tq = %d query rows per K/V head (at most %d)",
             (p->H / p->H_kv) * p->Tq, kDecMaxRows);
    return set_last_error(FA_ERR_UNSUPPORTED, msg);
  }
  if (p->Tq > p->Tkv) return set_last_error(FA_ERR_INVALID, "fa_decode: Tq > Tkv");
  if ((int64_t)p->B * p->H_kv > 65535) return set_last_error(FA_ERR_UNSUPPORTED, "fa_decode: B * H_kv > 65535");
  if (p->mask.flags & ~(FA_MASK_CAUSAL | FA_MASK_WINDOW))
    return set_last_error(FA_ERR_UNSUPPORTED, "fa_decode: only causal and sliding-window masks");
  if (p->mask.q_offset || p->mask.kv_offset)
    return set_last_error(FA_ERR_INVALID, "fa_decode: positions come from kv_lens; offsets must be 0");
  if (p->score.flags & ~(FA_SCORE_ALIBI | FA_SCORE_SOFTCAP))
    return set_last_error(FA_ERR_UNSUPPORTED, "fa_decode: only ALiBi and softcap score mods");
  if ((p->score.flags & FA_SCORE_ALIBI) && !p->score.alibi_slopes)
    return set_last_error(FA_ERR_INVALID, "fa_decode: ALiBi without slopes");
  if ((p->score.flags & FA_SCORE_SOFTCAP) && !(p->score.softcap > 0.f))
    return set_last_error(FA_ERR_INVALID, "fa_decode: softcap must be > 0");
  if (p->num_splits < 0) return set_last_error(FA_ERR_INVALID, "fa_decode: num_splits < 0");
  return FA_OK;
}

template <typename T, int D>
cudaError_t launch_split(const CUtensorMap& tk, const CUtensorMap& tv, const DecodeArgs& a, size_t smem,
                         cudaStream_t stream) {
  cudaError_t e =
      cudaFuncSetAttribute(decode_split_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  decode_split_kernel<T, D><<<dim3((unsigned)a.splits, (unsigned)(a.B * a.Hkv)), kDecThreads, smem, stream>>>(
      tk, tv, a);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_decode(const CUtensorMap& tk, const CUtensorMap& tv, const DecodeArgs& a, size_t smem,
                          cudaStream_t stream) {
  cudaError_t e = a.D == 64    ? launch_split<T, 64>(tk, tv, a, smem, stream)
                  : a.D == 128 ? launch_split<T, 128>(tk, tv, a, smem, stream)
                               : launch_split<T, 256>(tk, tv, a, smem, stream);
  if (e != cudaSuccess) return e;
  const int64_t rows = (int64_t)a.B * a.H * a.Tq;
  decode_merge_kernel<T><<<(unsigned)((rows + 7) / 8), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

size_t workspace_bytes_of(const FaDecodeParams* p, const DecodePlan& pl) {
  const size_t rows = (size_t)p->B * p->H * p->Tq;
  return (size_t)pl.splits * rows * ((size_t)p->D + 1) * sizeof(float) + 256;
}

}  // namespace
}  // namespace fa

extern "C" {

int fa_decode_workspace_size(const FaDecodeParams* p, size_t* bytes) {
  int rc = fa::check_decode(p);
  if (rc) return rc;
  if (!bytes) return fa::set_last_error(FA_ERR_INVALID, "fa_decode_workspace_size: bytes is NULL");
  *bytes = fa::workspace_bytes_of(p, fa::plan_decode(p));
  return FA_OK;
}

int fa_decode(const FaDecodeParams* p, void* workspace, size_t workspace_bytes, fa_stream_t stream) {
  int rc = fa::check_decode(p);
  if (rc) return rc;
  if (!p->q.ptr || !p->k.ptr || !p->v.ptr || !p->o.ptr || !p->lse)
    return fa::set_last_error(FA_ERR_INVALID, "fa_decode: NULL tensor");
  const fa::DecodePlan pl = fa::plan_decode(p);
  char msg[192];
  const size_t need = fa::workspace_bytes_of(p, pl);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15u)) {
    snprintf(msg, sizeof(msg), "fa_decode: workspace must be 16-byte aligned and hold %zu bytes", need);
    return fa::set_last_error(FA_ERR_INVALID, msg);
  }
  CUtensorMap tk, tv;
  if ((rc = fa::make_row_tile_map(&tk, p->k, p->dtype, p->B, p->H_kv, p->Tkv, p->D, fa::kDecKT, "k")) ||
      (rc = fa::make_row_tile_map(&tv, p->v, p->dtype, p->B, p->H_kv, p->Tkv, p->D, fa::kDecKT, "v")))
    return rc;
  fa::DecodeArgs a;
  a.B = p->B;
  a.H = p->H;
  a.Hkv = p->H_kv;
  a.Tq = p->Tq;
  a.Tkv = p->Tkv;
  a.D = p->D;
  a.G = p->H / p->H_kv;
  a.M = a.G * p->Tq;
  a.splits = pl.splits;
  a.chunk = pl.chunk;
  a.stages = pl.stages;
  a.q = p->q;
  a.o = p->o;
  a.lse = p->lse;
  a.kv_lens = p->kv_lens;
  a.scale = p->scale;
  a.mask = p->mask;
  a.score = p->score;
  const size_t rows = (size_t)p->B * p->H * p->Tq;
  a.part_o = reinterpret_cast<float*>(workspace);
  a.part_lse = a.part_o + (size_t)pl.splits * rows * p->D;
  a.status = p->status;
  cudaError_t e = p->dtype == FA_DTYPE_F32
                      ? fa::launch_decode<float>(tk, tv, a, pl.smem, (cudaStream_t)stream)
                      : fa::launch_decode<__nv_bfloat16>(tk, tv, a, pl.smem, (cudaStream_t)stream);
  if (e != cudaSuccess) {
    snprintf(msg, sizeof(msg), "fa_decode: %s", cudaGetErrorString(e));
    return fa::set_last_error(FA_ERR_CUDA, msg);
  }
  return FA_OK;
}

}  // extern "C"
