// Split-KV decode: a few new query tokens per sequence against a K/V cache (fa_decode).
//
// Decode reads the whole cache once per call and does O(G * Tq) multiply-adds per cache
// element, so with a handful of query rows it is bound by HBM bandwidth.  The cache of each
// (b, K/V head) is cut into num_splits chunks; one CTA per (chunk, b, K/V head) handles
// every query row of the K/V head's group (G = H / H_kv heads x Tq tokens = M rows), so each
// cache element is read from HBM once for all of them.  Query row i of batch b sits at
// global position kv_lens[b] - Tq + i.  Two split kernels:
//
// * decode_tc_kernel (bf16, M <= 128): tcgen05 MMAs with the query rows as the MMA's M; its
//   own comment below describes it.
// * decode_split_kernel (fp32, M <= 64), on CUDA cores.  Per CTA, TMA streams 64-row K and V
//   tiles (128-byte swizzled panels) through a ring of stages guarded by mbarriers; the 256
//   threads then run, per tile,
//     scores   thread = (cache row j, every 4th query row): 16-byte K chunks against fp32 Q
//              (the swizzle spreads the 32 rows a warp reads over all banks); with one or
//              two query rows the threads split the head dimension instead,
//     softmax  warp = query row, online (running max and sum per row),
//     P V      thread = (8 output columns, every RG-th query row), fp32 accumulators in
//              registers, probabilities read 4 cache rows at a time; with fewer query rows
//              than RG the threads also split the tile's cache rows (partials added at the end),
//   and thread 0 refills the stage.
//
// Each CTA writes its normalised partial (o, lse) to the workspace and decode_merge_kernel
// combines the chunks by log-sum-exp (the tcgen05 kernel writes o and lse itself when there
// is a single chunk).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>

#include "fa_common.cuh"
#include "fa_internal.h"
#include "fa_ptx.cuh"
#include "flexattn.h"

namespace fa {
namespace {

constexpr int kDecThreads = 256;
constexpr int kDecKT = 64;          // cache rows per tile (the TMA box height)
constexpr int kDecMaxRows = 64;     // G * Tq, CUDA-core kernel (fp32)
constexpr int kDecMaxRowsTc = 128;  // G * Tq, tcgen05 kernel (bf16)
constexpr int kDecPS = kDecKT + 4;  // row stride of the score tile in floats (16-byte aligned, bank-shifted)
constexpr int kPanelBytes = kDecKT * 128;

struct DecodeArgs {
  int B, H, Hkv, Tq, Tkv, D, G, M, splits, chunk, stages;
  int q_vec;  // q's base and strides are 16-byte multiples (the tcgen05 kernel loads 8 bf16 at once)
  int o_vec;  // the same for o (the tcgen05 kernel stores 8 bf16 at once when it writes o itself)
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

  // score phase: thread = (cache row jrow, row group mg); with M = 1 or 2 the groups split the
  // head dimension into DS parts instead, leaving MG = 4 / DS row groups
  const int jrow = tid % kDecKT, mg = tid / kDecKT;
  const int DS = M == 1 ? 4 : (M == 2 ? 2 : 1), MG = 4 / DS, ds = mg % DS, mq = mg / DS;
  // P V phase: thread = (column group cg, slot rg); with fewer rows than slots the slots also
  // split the tile's cache rows into JG groups (partial sums added at the end)
  const int cg = tid % NCG, rg = tid / NCG;
  int JG = 1;
  {
    int m2 = 1;
    while (m2 < M) m2 <<= 1;
    if (m2 < RG) JG = min(16, RG / m2);
  }
  const int RS = RG / JG, jg = rg / RS, mrow = rg % RS, jlen = kDecKT / JG;
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

    // ---- scores (log2 domain), masked to -inf.  With M < 4 the four row groups split the
    //      head dimension instead (DS parts); part ds > 0 leaves its partial dot product in
    //      score row ds * M + m for part 0 to add.
    {
      const int c0 = ds * (CHUNKS / DS), c1 = c0 + CHUNKS / DS;
      float dot[SPT];
#pragma unroll
      for (int r = 0; r < SPT; ++r) dot[r] = 0.f;
#pragma unroll 2
      for (int c = c0; c < c1; ++c) {
        float kf[EPC];
        unpack_chunk(*reinterpret_cast<const uint4*>(kst + chunk_off(jrow, c)), kf);
#pragma unroll
        for (int r = 0; r < SPT; ++r) {
          const int m = mq + MG * r;
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
      if (DS > 1) {
        if (ds > 0 && mq < M) sP[(ds * M + mq) * kDecPS + jrow] = dot[0];
        __syncthreads();
        if (ds == 0 && mq < M)
          for (int d2 = 1; d2 < DS; ++d2) dot[0] += sP[(d2 * M + mq) * kDecPS + jrow];
      }
      if (ds == 0) {
        const int kvpos = t0 + jrow;
#pragma unroll
        for (int r = 0; r < SPT; ++r) {
          const int m = mq + MG * r;
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
    // ---- P V over this thread's share of the tile's first n rows, rounded up to 4 (the rows
    //      past n are zero)
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
      const int m = mrow + RS * r;
      if (m < M) {
        const float al = sAlpha[m];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[r][e] *= al;
      }
    }
    for (int j0 = jg * jlen, j1 = min(j0 + jlen, n); j0 < j1; j0 += 4) {
      float4 p4[RPT];
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const int m = mrow + RS * r;
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
  if (JG > 1) {  // add the row groups' partial sums (row mrow only: RS >= M); the stages are free now
    float* red = reinterpret_cast<float*>(base);  // [JG][RS][D]
    __syncthreads();
    if (mrow < M) {
      float4* dst = reinterpret_cast<float4*>(red + (jg * RS + mrow) * D + cg * 8);
      dst[0] = make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]);
      dst[1] = make_float4(acc[0][4], acc[0][5], acc[0][6], acc[0][7]);
    }
    __syncthreads();
    if (jg == 0 && mrow < M)
      for (int g2 = 1; g2 < JG; ++g2) {
        const float4* src = reinterpret_cast<const float4*>(red + (g2 * RS + mrow) * D + cg * 8);
        const float4 lo = src[0], hi = src[1];
        acc[0][0] += lo.x; acc[0][1] += lo.y; acc[0][2] += lo.z; acc[0][3] += lo.w;
        acc[0][4] += hi.x; acc[0][5] += hi.y; acc[0][6] += hi.z; acc[0][7] += hi.w;
      }
  }
  // ---- this chunk's normalised partial (o, lse); an empty chunk gives o = 0, lse = -inf
  const int64_t rows = (int64_t)a.B * a.H * a.Tq;
#pragma unroll
  for (int r = 0; r < RPT; ++r) {
    const int m = mrow + RS * r;
    if (m >= M || jg != 0) continue;
    const int g = m / a.Tq, i = m % a.Tq;
    const int64_t row = ((int64_t)b * a.H + hk * a.G + g) * a.Tq + i;
    const float l = sSum[m], inv = l > 0.f ? 1.f / l : 0.f;
    float4* dst = reinterpret_cast<float4*>(a.part_o + ((int64_t)s * rows + row) * D + cg * 8);
    dst[0] = make_float4(acc[r][0] * inv, acc[r][1] * inv, acc[r][2] * inv, acc[r][3] * inv);
    dst[1] = make_float4(acc[r][4] * inv, acc[r][5] * inv, acc[r][6] * inv, acc[r][7] * inv);
    if (cg == 0) a.part_lse[(int64_t)s * rows + row] = l > 0.f ? (sMax[m] + log2f(l)) * kLn2 : -INFINITY;
  }
}

// ---------------------------------------------------------------------------------------------
// tcgen05 split kernel (bf16).  The query rows of the group (M <= 128, zero-padded to 128) are
// the MMA's M dimension and the KT-row cache tile its N:
//   S = Q K^T   (kind::f16, M = 128, N = KT, K = D; Q and K from shared memory) into one of two
//               TMEM score buffers, so the next tile's S is computed during this tile's softmax,
//   P = exp2(S - m) by the warps that own the rows (thread = row, as in the forward kernel),
//               written back over S in TMEM as bf16,
//   O += P V    (A = P from TMEM, B = V from shared memory, MN-major; N = D).
// The padded rows cost tensor-core time only, of which decode has plenty: a tile's HBM bytes
// take longer than its MMAs.  Warps: ceil(M / 32) softmax warps (those whose TMEM lanes hold
// real rows), one MMA-issue warp and one producer warp that streams K/V tiles through the
// stage ring, refilling a stage as soon as the PV MMA that read it completes (per-stage
// empty barriers committed by the MMA issuer).  The row max used for P moves only
// when a tile's max exceeds it by more than 8 (log2 units): O is rescaled rarely and P <= 256.
// With a single chunk (num_splits = 1) the CTA writes the final o and lse itself and no merge
// kernel runs.
constexpr float kDecRescaleThreshold = 8.f;

// Cache rows per tile of the tcgen05 kernel (the S MMA's N and the TMA box height).  A
// 128-row tile halves the per-tile fixed costs of the softmax warp (waits, TMEM round
// trips, barrier arrivals) at head dim 128; head dims 64 and 256 keep 64 rows (64: two CTAs
// per SM fit only with 64-row tiles; 256: shared memory holds two 64-row stages).
#ifndef FA_DEC_KT_D64
#define FA_DEC_KT_D64 64
#endif
#ifndef FA_DEC_KT_D128
#define FA_DEC_KT_D128 128
#endif
__host__ __device__ constexpr int decode_tc_kt(int D) {
  return D <= 64 ? FA_DEC_KT_D64 : (D <= 128 ? FA_DEC_KT_D128 : 64);
}

// TMEM columns: two S buffers of KT fp32 columns and O (D columns), rounded to a power of 2.
__host__ __device__ constexpr uint32_t decode_tc_tmem_cols(int D, int KT) { return 2 * KT + D <= 256 ? 256u : 512u; }

// Dynamic shared memory of the tcgen05 kernel: K/V stages, the 128-row Q operand, barriers.
inline size_t decode_tc_smem_bytes(int D, int stages) {
  return 1024 + (size_t)stages * 2 * decode_tc_kt(D) * D * 2 + (size_t)128 * D * 2 + 256;
}

// Byte offset of 16-byte chunk c of row r in a tile of 128-byte swizzled panels of PANEL
// bytes each (panel c / 8, chunk slot (c % 8) ^ (r % 8) of the row's 128-byte line).
template <int PANEL>
__device__ __forceinline__ uint32_t chunk_off_p(int r, int c) {
  return (uint32_t)((c >> 3) * PANEL + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// CTAs per SM of the tcgen05 kernel: as many as TMEM serves (512 columns), at most two.
// Head dim 64 with 64-row tiles: two (5 stages each), as a 16 KB tile gives one softmax
// chain too little time per byte (measured 5.0 vs 2.7 TB/s on B32 H16 Tkv8192).  Head dim
// 128 (128-row tiles) and 256: one.
inline int decode_tc_ctas_per_sm(int D) { return decode_tc_tmem_cols(D, decode_tc_kt(D)) <= 256 ? 2 : 1; }

__device__ __forceinline__ bool bar_red_or(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %3, 0;\n\t"
      "barrier.cta.red.or.pred q, %1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(nthreads), "r"((uint32_t)pred)
      : "memory");
  return r != 0;
}

template <int D, int KT>
__global__ void __launch_bounds__(192) decode_tc_kernel(const __grid_constant__ CUtensorMap tk,
                                                        const __grid_constant__ CUtensorMap tv, const DecodeArgs a) {
  constexpr int TILE = KT * D * 2;  // bytes of a KT-row K or V tile
  constexpr int PANELB = KT * 128;  // bytes of one 64-column panel of a tile
  constexpr int QPANEL = 128 * 128;     // bytes of one 64-column panel of the 128-row Q operand
  constexpr int NPANEL = D / 64;
  constexpr uint32_t TM_COLS = decode_tc_tmem_cols(D, KT);
  constexpr uint32_t TM_S = 0, TM_O = 2 * KT;  // S buffers at 0 and KT (fp32; P over them as bf16), O
  constexpr uint32_t IDESC_S = make_idesc_bf16(128, KT, 0, 0);
  constexpr uint32_t IDESC_PV = make_idesc_bf16(128, D, 0, 1);

  extern __shared__ unsigned char dsm_raw[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages, M = a.M;
  const int nw = (int)(blockDim.x >> 5) - 2;  // softmax warps; then the MMA warp and the producer warp
  const int nsm = 32 * nw;
  const int mma_warp = nw, prod_warp = nw + 1;
  unsigned char* sQ = base + (size_t)S * 2 * TILE;
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(sQ + NPANEL * QPANEL);  // [S] tile landed
  uint64_t* bar_empty = bar_full + S;                                      // [S] tile's MMAs retired
  uint64_t* bar_s = bar_empty + S;                                         // [2] S buffer computed
  uint64_t* bar_p = bar_s + 2;                                             // [2] P buffer written (nw arrivals)
  uint64_t* bar_o = bar_p + 2;                                             // PV retired (one phase per tile)
  uint64_t* bar_fin = bar_o + 1;                                           // all MMAs retired
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_fin + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* never = abort_flag + 1;  // stays 0: waits on it end by time only

  const int s = blockIdx.x, bhk = blockIdx.y, b = bhk / a.Hkv, hk = bhk % a.Hkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int len = a.kv_lens ? min(max(__ldg(a.kv_lens + b), 0), a.Tkv) : a.Tkv;
  const int kv0 = s * a.chunk, kv1 = min(kv0 + a.chunk, len);
  const int ntiles = kv1 > kv0 ? (kv1 - kv0 + KT - 1) / KT : 0;
  const int qbase = len - a.Tq;

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(bar_full + i, 1);
      mbar_init(bar_empty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_s + i, 1);
      mbar_init(bar_p + i, nw);
    }
    mbar_init(bar_o, 1);
    mbar_init(bar_fin, 1);
    *abort_flag = 0;
    *never = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, TM_COLS);
    tmem_relinquish();
  }
  __syncthreads();  // barriers initialised
  // The producer starts the first tiles' loads before the Q operand is built, so a short
  // chunk's first load overlaps the prologue.
  int issued = 0;  // producer lane 0: tiles whose loads were issued
  auto issue = [&](int t) {
    const int st = t % S;
    unsigned char* dst = base + (size_t)st * 2 * TILE;
    mbar_arrive_expect_tx(bar_full + st, 2 * TILE);
#pragma unroll
    for (int p = 0; p < NPANEL; ++p) {
      tma_load_4d(dst + p * PANELB, &tk, bar_full + st, p * 64, kv0 + t * KT, hk, b);
      tma_load_4d(dst + TILE + p * PANELB, &tv, bar_full + st, p * 64, kv0 + t * KT, hk, b);
    }
    issued = t + 1;
  };
  if (warp == prod_warp && lane == 0) {
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    for (int t = 0; t < min(S, ntiles); ++t) issue(t);
  }
  // Q operand: row m < M is query token (g, i) = (m / Tq, m % Tq) of head hk * G + g, other
  // rows zero; 128-byte swizzled 64-column panels (the TMA layout of the K tiles).  16-byte
  // loads when q's base and strides allow them.
  for (int e = tid; e < 128 * (D / 8); e += blockDim.x) {
    const int r = e / (D / 8), c = e % (D / 8);
    uint4 w = make_uint4(0u, 0u, 0u, 0u);
    if (r < M) {
      const uint16_t* qh = reinterpret_cast<const uint16_t*>(a.q.ptr) + (int64_t)b * a.q.stride_b +
                           (int64_t)(hk * a.G + r / a.Tq) * a.q.stride_h + (int64_t)(r % a.Tq) * a.q.stride_t +
                           c * 8;
      if (a.q_vec) {
        w = __ldg(reinterpret_cast<const uint4*>(qh));
      } else {
        w.x = (uint32_t)qh[0] | ((uint32_t)qh[1] << 16);
        w.y = (uint32_t)qh[2] | ((uint32_t)qh[3] << 16);
        w.z = (uint32_t)qh[4] | ((uint32_t)qh[5] << 16);
        w.w = (uint32_t)qh[6] | ((uint32_t)qh[7] << 16);
      }
    }
    *reinterpret_cast<uint4*>(sQ + (c >> 3) * QPANEL + r * 128 + (((c & 7) ^ (r & 7)) << 4)) = w;
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == prod_warp) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      for (int t = issued; t < ntiles; ++t) {
        const int st = t % S;
        if (t >= S && !mbar_wait(bar_empty + st, (uint32_t)(((t / S) - 1) & 1), abort_flag)) break;
        issue(t);
      }
      // every stage's latest load lands before the CTA may exit (earlier uses were consumed)
      for (int t = max(0, issued - S); t < issued; ++t)
        mbar_wait(bar_full + t % S, (uint32_t)((t / S) & 1), never);
    }
    __syncwarp();
  } else if (warp == mma_warp) {
    // ------------------------------------------------------------------ MMA issue
    // Order: S(0), S(1), then per tile PV(t) once its P is written, and S(t + 2) into the
    // buffer PV(t) has just read (the tensor pipe runs one issuer's MMAs in order).
    const uint32_t q_lo = (uint32_t)make_smem_desc(smem_u32(sQ), 16, 1024, SMEM_SWIZZLE_128B);
    const uint32_t desc_hi = (uint32_t)(make_smem_desc(smem_u32(sQ), 16, 1024, SMEM_SWIZZLE_128B) >> 32);
    const uint32_t k_lo0 = (uint32_t)make_smem_desc(smem_u32(base), 16, 1024, SMEM_SWIZZLE_128B);
    const uint32_t v_lo0 = (uint32_t)make_smem_desc(smem_u32(base), PANELB, 1024, SMEM_SWIZZLE_128B);
    auto issue_s = [&](int t) -> bool {
      const int st = t % S;
      if (!mbar_wait_w(bar_full + st, (uint32_t)((t / S) & 1), abort_flag)) return false;
      tc_fence_after();
      const uint32_t k_lo = k_lo0 + (uint32_t)((st * 2 * TILE) >> 4);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        mma_ss_w(tmem + TM_S + (t & 1) * KT, q_lo + (kk >> 2) * (QPANEL >> 4) + (kk & 3) * 2, desc_hi,
                 k_lo + (kk >> 2) * (PANELB >> 4) + (kk & 3) * 2, desc_hi, IDESC_S, kk > 0);
      tc_commit_w(bar_s + (t & 1));
      return true;
    };
    bool ok = true;
    for (int t = 0; t < min(2, ntiles) && ok; ++t) ok = issue_s(t);
    for (int it = 0; it < ntiles && ok; ++it) {
      const int st = it % S;
      if (!mbar_wait_w(bar_p + (it & 1), (uint32_t)((it >> 1) & 1), abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t v_lo = v_lo0 + (uint32_t)((st * 2 * TILE + TILE) >> 4);
#pragma unroll
      for (int kk = 0; kk < KT / 16; ++kk)
        mma_ts_w(tmem + TM_O, tmem + TM_S + (it & 1) * KT + kk * 8, v_lo + kk * (2048 >> 4), desc_hi,
                 IDESC_PV, (it > 0 || kk > 0) ? 1u : 0u);
      tc_commit_w(bar_empty + st);
      tc_commit_w(bar_o);
      if (it + 2 < ntiles) ok = issue_s(it + 2);
    }
    if (!ok && lane == 0) *abort_flag = 1;
    tc_commit_w(bar_fin);
  } else {
    // ------------------------------------------------------------------ softmax (thread = row)
    const uint32_t t_lane = tmem + ((uint32_t)(warp * 32) << 16);
    const int r = tid;
    const bool real = r < M;
    const int qpos = qbase + r % a.Tq;
    const float slope =
        (real && (a.score.flags & FA_SCORE_ALIBI)) ? a.score.alibi_slopes[hk * a.G + r / a.Tq] : 0.f;
    const bool softcap = (a.score.flags & FA_SCORE_SOFTCAP) != 0;
    const bool plain = !softcap && !(a.score.flags & FA_SCORE_ALIBI);
    const float cap = softcap ? a.score.softcap : 1.f, inv_cap = 1.f / cap;
    int lo = 0, hi = real ? len - 1 : -1;  // allowed cache positions of this row
    if (a.mask.flags & FA_MASK_CAUSAL) hi = min(hi, qpos);
    if (a.mask.flags & FA_MASK_WINDOW) {
      if (a.mask.window_left >= 0) lo = max(lo, qpos - a.mask.window_left);
      if (a.mask.window_right >= 0) hi = min(hi, qpos + a.mask.window_right);
    }
    const float k_log2 = a.scale * kLog2e;

    float m_use = -INFINITY, l_run = 0.f;
    for (int it = 0; it < ntiles; ++it) {
      const int st = it % S, t0 = kv0 + it * KT, n = min(KT, kv1 - t0);
      const uint32_t tS = t_lane + TM_S + (it & 1) * KT;
      const bool got = mbar_wait(bar_s + (it & 1), (uint32_t)((it >> 1) & 1), abort_flag);
      if (bar_red_or(1, nsm, !got)) {
        if (tid == 0) *abort_flag = 1;  // the MMA and producer warps stop waiting too
        break;
      }
      tc_fence_after();
      float x[KT];
      {
        uint32_t rr[KT / 32][32];
#pragma unroll
        for (int h = 0; h < KT / 32; ++h) tmem_ld32(tS + 32 * h, rr[h]);
        tmem_ld_wait();
#pragma unroll
        for (int h = 0; h < KT / 32; ++h) {
          reg_pin(rr[h]);
#pragma unroll
          for (int c = 0; c < 32; ++c) x[32 * h + c] = __uint_as_float(rr[h][c]);
        }
      }
      // Rows whose every key of the tile is allowed (and padding rows, whose values are
      // never used) keep raw logits when the whole warp can: the max is taken on them and
      // the scale folds into the exponent's FMA.  Otherwise x becomes the masked
      // log2-domain logit.
      const bool inside = !real || (lo <= t0 && t0 + KT - 1 <= hi);
      const bool fast = plain && __all_sync(0xffffffffu, inside);
      if (!fast) {
#pragma unroll
        for (int c = 0; c < KT; ++c) {
          const int kv = t0 + c;
          float sc = fmaf(slope, (float)(kv - qpos), x[c] * a.scale);
          if (softcap) sc = cap * fast_tanh(sc * inv_cap);
          x[c] = (kv >= lo && kv <= hi) ? sc * kLog2e : -INFINITY;
        }
      }
      float m8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) m8[k] = fmax3f(x[k], x[8 + k], x[16 + k]);
#pragma unroll
      for (int c = 24; c < KT; c += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = fmax3f(m8[k], x[c + k], c + 8 + k < KT ? x[c + 8 + k] : -INFINITY);
      float mx = fmax3f(fmax3f(m8[0], m8[1], m8[2]), fmax3f(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
      if (fast) mx *= k_log2;  // k_log2 > 0
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m_use + kDecRescaleThreshold) {  // also the first finite max (m_use = -inf)
        if (m_use != -INFINITY) {               // O holds earlier tiles' sums at the old reference
          alpha = ex2_approx(m_use - mx);
          rescale = true;
        }
        m_use = mx;
      }
      if (__any_sync(0xffffffffu, rescale)) {
        // PV(it - 1) must have retired before O is touched
        if (it > 0 && !mbar_wait(bar_o, (uint32_t)((it - 1) & 1), abort_flag)) {
          if (lane == 0) *abort_flag = 1;
        } else {
          tc_fence_after();
#pragma unroll 1
          for (int c0 = 0; c0 < D; c0 += 32) {
            uint32_t ov[32];
            tmem_ld32(t_lane + TM_O + c0, ov);
            tmem_ld_wait();
            reg_pin(ov);
#pragma unroll
            for (int c = 0; c < 32; ++c) ov[c] = __float_as_uint(__uint_as_float(ov[c]) * alpha);
            tmem_st32(t_lane + TM_O + c0, ov);
          }
        }
      }
      l_run *= alpha;
      const float mref = m_use == -INFINITY ? 0.f : m_use;
      const float kk = fast ? k_log2 : 1.f;
      const float2 k2 = make_float2(kk, kk), nm2 = make_float2(-mref, -mref);
      float2 sum2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int h = 0; h < KT / 64; ++h) {
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 64; c += 2) {
          const float2 y = __ffma2_rn(make_float2(x[64 * h + c], x[64 * h + c + 1]), k2, nm2);
          const float2 p = make_float2(ex2_approx(y.x), ex2_approx(y.y));
          sum2[(c >> 1) & 3] = __fadd2_rn(sum2[(c >> 1) & 3], p);
          pk[c >> 1] = pack_bf16x2(p.x, p.y);
        }
        tmem_st32(tS + 32 * h, pk);
      }
      const float2 s01 = __fadd2_rn(sum2[0], sum2[1]), s23 = __fadd2_rn(sum2[2], sum2[3]);
      const float2 s4 = __fadd2_rn(s01, s23);
      l_run += s4.x + s4.y;
      if (n < KT) {  // tile rows past the chunk's end hold other data: zero them in V
        unsigned char* vst = base + (size_t)st * 2 * TILE + TILE;
        for (int e = tid; e < (KT - n) * (D / 8); e += nsm)
          *reinterpret_cast<uint4*>(vst + chunk_off_p<PANELB>(n + e / (D / 8), e % (D / 8))) = make_uint4(0, 0, 0, 0);
        fence_proxy_async_smem();
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_p + (it & 1));
    }
    // ---- wait for the last MMAs (also after an abort), then the epilogue
    const bool fin = mbar_wait(bar_fin, 0, never);
    const bool good = fin && !*abort_flag;
    if (!good && tid == 0) report_status(a.status, FA_ERR_TIMEOUT);
    tc_fence_after();
    const int64_t rows = (int64_t)a.B * a.H * a.Tq;
    const int64_t row = ((int64_t)b * a.H + hk * a.G + r / a.Tq) * a.Tq + r % a.Tq;
    const bool have_o = good && ntiles > 0;
    const bool live = have_o && l_run > 0.f;
    const float inv = live ? 1.f / l_run : 0.f;
#pragma unroll 1
    for (int c0 = 0; c0 < D; c0 += 32) {
      uint32_t ov[32];
      if (have_o) {
        tmem_ld32(t_lane + TM_O + c0, ov);
        tmem_ld_wait();
        reg_pin(ov);
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) ov[c] = 0u;
      }
      if (real && good && a.splits == 1) {  // one chunk: the final o, no merge
        uint16_t* orow = reinterpret_cast<uint16_t*>(a.o.ptr) + (int64_t)b * a.o.stride_b +
                         (int64_t)(hk * a.G + r / a.Tq) * a.o.stride_h + (int64_t)(r % a.Tq) * a.o.stride_t + c0;
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2)
          pk[c >> 1] = pack_bf16x2(__uint_as_float(ov[c]) * inv, __uint_as_float(ov[c + 1]) * inv);
        if (a.o_vec) {
#pragma unroll
          for (int v = 0; v < 4; ++v)
            reinterpret_cast<uint4*>(orow)[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        } else {
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            orow[2 * c] = (uint16_t)(pk[c] & 0xffffu);
            orow[2 * c + 1] = (uint16_t)(pk[c] >> 16);
          }
        }
      } else if (real && good) {
        float4* dst = reinterpret_cast<float4*>(a.part_o + ((int64_t)s * rows + row) * D + c0);
#pragma unroll
        for (int v = 0; v < 8; ++v)
          dst[v] = make_float4(__uint_as_float(ov[4 * v]) * inv, __uint_as_float(ov[4 * v + 1]) * inv,
                               __uint_as_float(ov[4 * v + 2]) * inv, __uint_as_float(ov[4 * v + 3]) * inv);
      }
    }
    if (real && good) {
      const float lse = live ? (m_use + __log2f(l_run)) * kLn2 : -INFINITY;
      if (a.splits == 1) a.lse[row] = lse;
      else a.part_lse[(int64_t)s * rows + row] = lse;
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
  }
}

// One warp per output row: log-sum-exp merge of the chunks' partials into o and lse.  The
// lanes first stride over the chunks for the max and the weights exp(lse_s - max) (kept in
// shared memory), then over the head dimension, summing the weighted partials chunk by chunk.
constexpr int kMaxSplits = 256;

template <typename T, int D>
__global__ void __launch_bounds__(256) decode_merge_kernel(const DecodeArgs a) {
  __shared__ float w_sh[8][kMaxSplits];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)a.B * a.H * a.Tq;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (row >= rows) return;
  float* w = w_sh[warp];
  float L = -INFINITY;
  for (int s = lane; s < a.splits; s += 32) L = fmaxf(L, a.part_lse[(int64_t)s * rows + row]);
#pragma unroll
  for (int o = 16; o; o >>= 1) L = fmaxf(L, __shfl_xor_sync(0xffffffffu, L, o));
  float wsum = 0.f;
  for (int s = lane; s < a.splits; s += 32) {
    const float ls = a.part_lse[(int64_t)s * rows + row];
    const float ws = ls == -INFINITY ? 0.f : expf(ls - L);
    w[s] = ws;
    wsum += ws;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
  __syncwarp();
  float acc[D / 32];
#pragma unroll
  for (int j = 0; j < D / 32; ++j) acc[j] = 0.f;
  const float* po = a.part_o + row * D + lane;
#pragma unroll 4
  for (int s = 0; s < a.splits; ++s) {
    const float ws = w[s];
#pragma unroll
    for (int j = 0; j < D / 32; ++j) acc[j] = fmaf(ws, po[(int64_t)s * rows * D + 32 * j], acc[j]);
  }
  const int i = (int)(row % a.Tq), bh = (int)(row / a.Tq), b = bh / a.H, h = bh % a.H;
  T* o = reinterpret_cast<T*>(a.o.ptr) + (int64_t)b * a.o.stride_b + (int64_t)h * a.o.stride_h +
         (int64_t)i * a.o.stride_t;
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
  for (int j = 0; j < D / 32; ++j) {
    if constexpr (sizeof(T) == 4) o[lane + 32 * j] = acc[j] * inv;
    else o[lane + 32 * j] = __float2bfloat16_rn(acc[j] * inv);
  }
  if (lane == 0) a.lse[row] = wsum > 0.f ? L + logf(wsum) : -INFINITY;
}

// Chunking and pipeline depth for a call.
struct DecodePlan {
  int splits, chunk, stages, threads;
  bool tc;  // tcgen05 kernel (bf16) or the CUDA-core kernel (fp32)
  size_t smem;
};

DecodePlan plan_decode(const FaDecodeParams* p) {
  DecodePlan pl;
  const int es = p->dtype == FA_DTYPE_F32 ? 4 : 2;
  const int M = (p->H / p->H_kv) * p->Tq;
  int sp = p->num_splits;
  if (sp <= 0) {
    // Chunks of at least 256 cache rows.  The tcgen05 kernel: take the smallest chunk count
    // whose grid fills its last wave (148 SMs x CTAs per SM) to >= 85 % (the most filled one
    // if none does, up to four waves).  The CUDA-core kernel: about four CTAs per SM.
    const int pairs = p->B * p->H_kv;
    const int max_sp = std::max(1, std::min(kMaxSplits, (p->Tkv + 255) / 256));
    if (p->dtype == FA_DTYPE_BF16) {
      const double slots = 148.0 * decode_tc_ctas_per_sm(p->D);
      int best = 1;
      double best_eff = -1.0;
      for (int c = 1; c <= max_sp; ++c) {
        const double waves = (double)pairs * c / slots;
        if (waves > 4.0 && c > 1) break;
        const double eff = waves / std::ceil(waves);
        if (eff > best_eff + 1e-9) {
          best_eff = eff;
          best = c;
        }
        if (eff >= 0.85) break;
      }
      sp = best;
    } else {
      sp = std::min(max_sp, std::max(1, (4 * 148 + pairs - 1) / pairs));
    }
  }
  if (sp > kMaxSplits) sp = kMaxSplits;
  if (sp > p->Tkv) sp = p->Tkv;
  const int kt = p->dtype == FA_DTYPE_BF16 ? decode_tc_kt(p->D) : kDecKT;
  int ch = (p->Tkv + sp - 1) / sp;
  ch = (ch + kt - 1) / kt * kt;  // chunks start on tile boundaries
  pl.chunk = ch;
  pl.splits = (p->Tkv + ch - 1) / ch;
  if (p->dtype == FA_DTYPE_BF16) {
    // tcgen05 kernel: as many CTAs per SM as TMEM holds (512 columns / the CTA's allocation),
    // 2..4 stages in that share of the 228 KB of shared memory, and never less shared memory
    // than keeps one more CTA out (an SM must not host more CTAs than TMEM serves at once).
    // Stages: as many (2..8) as the CTA's share of the SM's 228 KB of shared memory holds; a
    // tile's load takes microseconds under load, so several must be in flight per SM.  The
    // request never falls below what keeps one more CTA out (TMEM holds 512 columns per SM).
    const int per_sm = decode_tc_ctas_per_sm(p->D);
    const size_t sm_total = 233472, reserved = 1024, max_dyn = 232448;
    const size_t budget = std::min(max_dyn, sm_total / per_sm - reserved);
    const size_t fixed = decode_tc_smem_bytes(p->D, 0), stage = decode_tc_smem_bytes(p->D, 1) - fixed;
    int S = (int)((budget - fixed) / stage);
    S = std::max(2, std::min(8, S));
    size_t smem = decode_tc_smem_bytes(p->D, S);
    const size_t floor_bytes = sm_total / (per_sm + 1) - reserved + 1;
    if (smem < floor_bytes) smem = floor_bytes;
    pl.stages = S;
    pl.smem = smem;
    pl.threads = 32 * ((M + 31) / 32) + 64;  // softmax warps, the MMA warp, the producer warp
    pl.tc = true;
    return pl;
  }
  // CUDA-core kernel (fp32): as many stages (<= 4) as leave room for two CTAs per SM; else
  // two, else one
  const size_t fixed = decode_smem_bytes(p->D, es, M, 0), stage = decode_smem_bytes(p->D, es, M, 1) - fixed;
  const size_t two_ctas = 113 * 1024, one_cta = 220 * 1024;
  int S = fixed + stage <= two_ctas ? (int)((two_ctas - fixed) / stage) : (fixed + 2 * stage <= one_cta ? 2 : 1);
  if (S > 4) S = 4;
  pl.stages = S;
  pl.smem = decode_smem_bytes(p->D, es, M, S);
  pl.threads = kDecThreads;
  pl.tc = false;
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
  const int max_rows = p->dtype == FA_DTYPE_BF16 ? kDecMaxRowsTc : kDecMaxRows;
  if ((int64_t)(p->H / p->H_kv) * p->Tq > max_rows) {
    snprintf(msg, sizeof(msg), "fa_decode: H / H_kv * Tq = %lld query rows per K/V head (at most %d for this dtype)",
             (long long)(p->H / p->H_kv) * p->Tq, max_rows);
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

template <int D>
cudaError_t launch_tc(const CUtensorMap& tk, const CUtensorMap& tv, const DecodeArgs& a, const DecodePlan& pl,
                      cudaStream_t stream) {
  constexpr int KT = decode_tc_kt(D);
  cudaError_t e =
      cudaFuncSetAttribute(decode_tc_kernel<D, KT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
  if (e != cudaSuccess) return e;
  decode_tc_kernel<D, KT>
      <<<dim3((unsigned)a.splits, (unsigned)(a.B * a.Hkv)), pl.threads, pl.smem, stream>>>(tk, tv, a);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_decode(const CUtensorMap& tk, const CUtensorMap& tv, const DecodeArgs& a, const DecodePlan& pl,
                          cudaStream_t stream) {
  cudaError_t e;
  if constexpr (sizeof(T) == 2) {
    e = a.D == 64    ? launch_tc<64>(tk, tv, a, pl, stream)
        : a.D == 128 ? launch_tc<128>(tk, tv, a, pl, stream)
                     : launch_tc<256>(tk, tv, a, pl, stream);
  } else {
    e = a.D == 64    ? launch_split<T, 64>(tk, tv, a, pl.smem, stream)
        : a.D == 128 ? launch_split<T, 128>(tk, tv, a, pl.smem, stream)
                     : launch_split<T, 256>(tk, tv, a, pl.smem, stream);
  }
  if (e != cudaSuccess) return e;
  if (sizeof(T) == 2 && a.splits == 1) return cudaSuccess;  // the tcgen05 kernel wrote o and lse
  const int64_t rows = (int64_t)a.B * a.H * a.Tq;
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  if (a.D == 64) decode_merge_kernel<T, 64><<<blocks, 256, 0, stream>>>(a);
  else if (a.D == 128) decode_merge_kernel<T, 128><<<blocks, 256, 0, stream>>>(a);
  else decode_merge_kernel<T, 256><<<blocks, 256, 0, stream>>>(a);
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
  const int box_rows = pl.tc ? fa::decode_tc_kt(p->D) : fa::kDecKT;
  if ((rc = fa::make_row_tile_map(&tk, p->k, p->dtype, p->B, p->H_kv, p->Tkv, p->D, box_rows, "k")) ||
      (rc = fa::make_row_tile_map(&tv, p->v, p->dtype, p->B, p->H_kv, p->Tkv, p->D, box_rows, "v")))
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
  a.q_vec = (reinterpret_cast<uintptr_t>(p->q.ptr) % 16 == 0) && (p->q.stride_b * 2) % 16 == 0 &&
            (p->q.stride_h * 2) % 16 == 0 && (p->q.stride_t * 2) % 16 == 0;
  a.o = p->o;
  a.o_vec = (reinterpret_cast<uintptr_t>(p->o.ptr) % 16 == 0) && (p->o.stride_b * 2) % 16 == 0 &&
            (p->o.stride_h * 2) % 16 == 0 && (p->o.stride_t * 2) % 16 == 0;
  a.lse = p->lse;
  a.kv_lens = p->kv_lens;
  a.scale = p->scale;
  a.mask = p->mask;
  a.score = p->score;
  const size_t rows = (size_t)p->B * p->H * p->Tq;
  a.part_o = reinterpret_cast<float*>(workspace);
  a.part_lse = a.part_o + (size_t)pl.splits * rows * p->D;
  a.status = p->status;
  cudaError_t e = p->dtype == FA_DTYPE_F32 ? fa::launch_decode<float>(tk, tv, a, pl, (cudaStream_t)stream)
                                           : fa::launch_decode<__nv_bfloat16>(tk, tv, a, pl, (cudaStream_t)stream);
  if (e != cudaSuccess) {
    snprintf(msg, sizeof(msg), "fa_decode: %s", cudaGetErrorString(e));
    return fa::set_last_error(FA_ERR_CUDA, msg);
  }
  return FA_OK;
}

}  // extern "C"
