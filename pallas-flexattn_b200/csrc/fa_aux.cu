// HBM-bound helper kernels of the backward pass and the context-parallel ring.
//
//   bwd_preprocess  delta = rowsum(O * dO) in fp32 (reference:
//                   flash_attention_bwd_preprocess_kernel, src/pallas_flexattn/
//                   flash_attn.py:168-173, which stores it in O's dtype) and
//                   lse2 = lse * log2(e); the same kernel zeroes the fp32 dQ
//                   accumulator (a memset on the same stream for the generic shapes).
//   dq_convert      dQ = scale * dq_accum, cast to the input dtype.
//   lse_merge       combine two partial (O, logsumexp) results over disjoint keys.
// bf16 rows of 64 or 128 elements (16-byte aligned) take the vector kernels: a few
// lanes per row, 16-byte loads, several rows per warp with every load issued before
// the first use.  Other shapes take one warp per row.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "fa_common.cuh"
#include "fa_internal.h"

namespace fa {
namespace {

constexpr int kRowsPerCta = 8;

template <typename T>
__device__ __forceinline__ float ldf(const T* p);
template <>
__device__ __forceinline__ float ldf<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// One warp per row of the padded [B*H, Tq_pad] grid.  Rows past Tq get delta = 0
// and lse2 = +inf (so exp2(x - lse2) = 0 there); rows with lse = -inf (no key)
// also get lse2 = +inf.
template <typename T>
__global__ void __launch_bounds__(kRowsPerCta * 32) preprocess_kernel(const AttnArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t prow = (int64_t)blockIdx.x * kRowsPerCta + warp;  // over B*H*Tq_pad
  const int64_t prows = (int64_t)a.B * a.H * a.Tq_pad;
  if (prow >= prows) return;
  const int t = (int)(prow % a.Tq_pad);
  const int bh = (int)(prow / a.Tq_pad), b = bh / a.H, h = bh % a.H;
  if (t >= a.Tq) {
    if (lane == 0) {
      a.delta[prow] = 0.f;
      if (a.lse2) a.lse2[prow] = INFINITY;
    }
    return;
  }
  const int64_t row = (int64_t)bh * a.Tq + t;
  const T* o = reinterpret_cast<const T*>(a.o.ptr) + (int64_t)b * a.o.stride_b + (int64_t)h * a.o.stride_h +
               (int64_t)t * a.o.stride_t;
  const T* g = reinterpret_cast<const T*>(a.dout.ptr) + (int64_t)b * a.dout.stride_b +
               (int64_t)h * a.dout.stride_h + (int64_t)t * a.dout.stride_t;
  float acc = 0.f;
  constexpr int V = 16 / sizeof(T);
  const bool vec = (a.D % V == 0) && ((reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(g)) % 16 == 0);
  if (vec) {
    for (int d0 = lane * V; d0 < a.D; d0 += 32 * V) {
      const uint4 ov = *reinterpret_cast<const uint4*>(o + d0);
      const uint4 gv = *reinterpret_cast<const uint4*>(g + d0);
      const T* op = reinterpret_cast<const T*>(&ov);
      const T* gp = reinterpret_cast<const T*>(&gv);
#pragma unroll
      for (int u = 0; u < V; ++u) acc = fmaf(ldf(op + u), ldf(gp + u), acc);
    }
  } else {
    for (int d = lane; d < a.D; d += 32) acc = fmaf(ldf(o + d), ldf(g + d), acc);
  }
#pragma unroll
  for (int s = 16; s; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
  if (lane == 0) {
    a.delta[prow] = acc;
    if (a.lse2) {
      const float l = a.lse_in[row];
      a.lse2[prow] = (l == -INFINITY) ? INFINITY : l * kLog2e;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kRowsPerCta * 32) dq_convert_kernel(const AttnArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kRowsPerCta + warp;
  const int64_t rows = (int64_t)a.B * a.H * a.Tq;
  if (row >= rows) return;
  const int t = (int)(row % a.Tq);
  const int bh = (int)(row / a.Tq), b = bh / a.H, h = bh % a.H;
  T* dq = reinterpret_cast<T*>(a.dq.ptr) + (int64_t)b * a.dq.stride_b + (int64_t)h * a.dq.stride_h +
          (int64_t)t * a.dq.stride_t;
  const float* src = a.dq_accum + row * a.D;
  for (int d = lane; d < a.D; d += 32) {
    const float x = src[d] * a.scale;
    if constexpr (sizeof(T) == 4) dq[d] = x;
    else dq[d] = __float2bfloat16_rn(x);
  }
}

template <typename T>
__global__ void __launch_bounds__(kRowsPerCta * 32)
    lse_merge_kernel(int rows, int D, float* o_acc, float* lse_acc, const T* o_part, int64_t stride,
                     const float* lse_part) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kRowsPerCta + warp;
  if (row >= rows) return;
  const float la = lse_acc[row], lb = lse_part[row];
  const float mx = fmaxf(la, lb);
  if (mx == -INFINITY) return;  // both empty: keep o_acc = 0, lse = -inf
  const float wa = (la == -INFINITY) ? 0.f : expf(la - mx);
  const float wb = (lb == -INFINITY) ? 0.f : expf(lb - mx);
  const float tot = wa + wb;
  const float ca = wa / tot, cb = wb / tot;
  float* oa = o_acc + row * D;
  const T* ob = o_part + row * stride;
  for (int d = lane; d < D; d += 32) oa[d] = oa[d] * ca + ldf(ob + d) * cb;
  if (lane == 0) lse_acc[row] = mx + logf(tot);
}

// Vector combine for bf16 parts of D = 64 or 128 (the ring's partial outputs): L = D / 8 lanes
// per row, a 16-byte load of the part and two of the fp32 accumulator per lane, kMergePasses
// rows per lane group with every load issued before the first use (the row-per-warp kernel
// above waits for the two logsumexps before it loads the row).
constexpr int kMergePasses = 4;

template <int D>
__global__ void __launch_bounds__(256)
    lse_merge_bf16_vec_kernel(int rows, float* o_acc, float* lse_acc, const __nv_bfloat16* o_part, int64_t stride,
                              const float* lse_part) {
  constexpr int L = D / 8;     // lanes per row
  constexpr int RPW = 32 / L;  // rows per warp and pass
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / L, c = (lane % L) * 8;
  const int64_t base = ((int64_t)blockIdx.x * 8 + warp) * (RPW * kMergePasses) + sub;
  float la[kMergePasses], lb[kMergePasses];
  uint4 pb[kMergePasses];
  float4 a0[kMergePasses], a1[kMergePasses];
#pragma unroll
  for (int k = 0; k < kMergePasses; ++k) {
    const int64_t row = base + k * RPW;
    la[k] = lb[k] = -INFINITY;
    if (row < rows) {
      la[k] = lse_acc[row];
      lb[k] = lse_part[row];
      pb[k] = *reinterpret_cast<const uint4*>(o_part + row * stride + c);
      a0[k] = *reinterpret_cast<const float4*>(o_acc + row * D + c);
      a1[k] = *reinterpret_cast<const float4*>(o_acc + row * D + c + 4);
    }
  }
#pragma unroll
  for (int k = 0; k < kMergePasses; ++k) {
    const int64_t row = base + k * RPW;
    const float mx = fmaxf(la[k], lb[k]);
    if (row >= rows || mx == -INFINITY) continue;  // both empty: keep o_acc = 0, lse = -inf
    const float wa = (la[k] == -INFINITY) ? 0.f : expf(la[k] - mx);
    const float wb = (lb[k] == -INFINITY) ? 0.f : expf(lb[k] - mx);
    const float tot = wa + wb;
    const float ca = wa / tot, cb = wb / tot;
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&pb[k]);
    const float2 b0 = __bfloat1622float2(h[0]), b1 = __bfloat1622float2(h[1]), b2 = __bfloat1622float2(h[2]),
                 b3 = __bfloat1622float2(h[3]);
    const float4 r0 = make_float4(a0[k].x * ca + b0.x * cb, a0[k].y * ca + b0.y * cb, a0[k].z * ca + b1.x * cb,
                                  a0[k].w * ca + b1.y * cb);
    const float4 r1 = make_float4(a1[k].x * ca + b2.x * cb, a1[k].y * ca + b2.y * cb, a1[k].z * ca + b3.x * cb,
                                  a1[k].w * ca + b3.y * cb);
    *reinterpret_cast<float4*>(o_acc + row * D + c) = r0;
    *reinterpret_cast<float4*>(o_acc + row * D + c + 4) = r1;
    if (lane % L == 0) lse_acc[row] = mx + logf(tot);
  }
}

constexpr int kVecPasses = 4;  // rows per lane group in flight

// Vector preprocess for bf16 rows of D = 64 or 128, fused with the zeroing of the fp32 dQ
// accumulator.  One CTA per (64-row block, b*h): no per-row index division, every load of
// the block issued before the first use (L = D / 8 lanes per row, 16 bytes each), delta and
// lse2 staged in shared memory and stored as two coalesced 256-byte rows, and the block's
// accumulator rows [bh, t0 .. t0+63, :] zeroed with coalesced 16-byte stores.  HBM traffic
// per row: reads 2*D*2 bytes (o, dO) + 4 (lse), writes D*4 (zeros) + 8 (delta, lse2).
constexpr int kPreRows = 64;

template <int D>
__global__ void __launch_bounds__(256) preprocess_bf16_zero_kernel(const AttnArgs a) {
  constexpr int L = D / 8, RPP = 256 / L, NP = kPreRows / RPP;
  __shared__ float s_delta[kPreRows];
  __shared__ float s_lse[kPreRows];
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int t0 = blockIdx.x * kPreRows;
  const int tid = threadIdx.x, sub = tid / L, li = tid % L;
  const __nv_bfloat16* obase = reinterpret_cast<const __nv_bfloat16*>(a.o.ptr) + (int64_t)b * a.o.stride_b +
                               (int64_t)h * a.o.stride_h + li * 8;
  const __nv_bfloat16* gbase = reinterpret_cast<const __nv_bfloat16*>(a.dout.ptr) + (int64_t)b * a.dout.stride_b +
                               (int64_t)h * a.dout.stride_h + li * 8;
  uint4 ov[NP], gv[NP];
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    const int t = t0 + p * RPP + sub;
    ov[p] = gv[p] = make_uint4(0u, 0u, 0u, 0u);
    if (t < a.Tq) {
      ov[p] = __ldg(reinterpret_cast<const uint4*>(obase + (int64_t)t * a.o.stride_t));
      gv[p] = __ldg(reinterpret_cast<const uint4*>(gbase + (int64_t)t * a.dout.stride_t));
    }
  }
  if (a.lse2 && tid < kPreRows) {
    const int t = t0 + tid;
    s_lse[tid] = t < a.Tq ? __ldg(a.lse_in + (int64_t)bh * a.Tq + t) : -INFINITY;
  }
  // zero the block's rows of the dQ accumulator ([B*H, Tq, D]; rows past Tq do not exist)
  {
    const int nrows = min(kPreRows, a.Tq - t0);
    if (nrows > 0) {
      float4* z = reinterpret_cast<float4*>(a.dq_accum + ((int64_t)bh * a.Tq + t0) * D);
      const int n4 = nrows * (D / 4);
      for (int i = tid; i < n4; i += 256) z[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    const __nv_bfloat162* o2 = reinterpret_cast<const __nv_bfloat162*>(&ov[p]);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv[p]);
    float acc = 0.f;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 of = __bfloat1622float2(o2[u]), gf = __bfloat1622float2(g2[u]);
      acc = fmaf(of.x, gf.x, fmaf(of.y, gf.y, acc));
    }
#pragma unroll
    for (int off = L / 2; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (li == 0) s_delta[p * RPP + sub] = acc;  // 0 for rows past Tq (their loads were zeros)
  }
  __syncthreads();
  if (tid < kPreRows) {
    const int t = t0 + tid;
    if (t < a.Tq_pad) a.delta[(int64_t)bh * a.Tq_pad + t] = s_delta[tid];
  } else if (a.lse2 && tid < 2 * kPreRows) {
    const int r = tid - kPreRows, t = t0 + r;
    const float l = s_lse[r];
    if (t < a.Tq_pad) a.lse2[(int64_t)bh * a.Tq_pad + t] = (l == -INFINITY) ? INFINITY : l * kLog2e;
  }
}

// Vector dQ conversion for bf16 output rows of D = 64 or 128: L = D / 4 lanes per row
// (16 bytes of fp32 in, 8 bytes of bf16 out each).
template <int D>
__global__ void __launch_bounds__(256) dq_convert_bf16_vec_kernel(const AttnArgs a) {
  constexpr int L = D / 4, RPP = 32 / L, RPW = RPP * kVecPasses;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / L, li = lane % L;
  const int64_t rows = (int64_t)a.B * a.H * a.Tq;
  const int64_t row0 = ((int64_t)blockIdx.x * 8 + warp) * RPW;
  float4 v[kVecPasses];
#pragma unroll
  for (int p = 0; p < kVecPasses; ++p) {
    const int64_t row = row0 + p * RPP + sub;
    v[p] = row < rows ? *reinterpret_cast<const float4*>(a.dq_accum + row * D + li * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int p = 0; p < kVecPasses; ++p) {
    const int64_t row = row0 + p * RPP + sub;
    if (row >= rows) continue;
    const int t = (int)(row % a.Tq);
    const int bh = (int)(row / a.Tq), b = bh / a.H, h = bh % a.H;
    __nv_bfloat16* dq = reinterpret_cast<__nv_bfloat16*>(a.dq.ptr) + (int64_t)b * a.dq.stride_b +
                        (int64_t)h * a.dq.stride_h + (int64_t)t * a.dq.stride_t + li * 4;
    const __nv_bfloat162 lo = __floats2bfloat162_rn(v[p].x * a.scale, v[p].y * a.scale);
    const __nv_bfloat162 hi = __floats2bfloat162_rn(v[p].z * a.scale, v[p].w * a.scale);
    uint2 w;
    w.x = *reinterpret_cast<const uint32_t*>(&lo);
    w.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(dq) = w;
  }
}

bool rows16(const FaTensor& t, int elem_bytes) {
  return (reinterpret_cast<uintptr_t>(t.ptr) % 16 == 0) && ((t.stride_t * elem_bytes) % 16 == 0) &&
         ((t.stride_h * elem_bytes) % 16 == 0) && ((t.stride_b * elem_bytes) % 16 == 0);
}

}  // namespace

cudaError_t launch_bwd_preprocess(const AttnArgs& a, int dtype, cudaStream_t stream) {
  const int64_t rows = (int64_t)a.B * a.H * a.Tq_pad;
  const bool vec = dtype == FA_DTYPE_BF16 && (a.D == 64 || a.D == 128) && rows16(a.o, 2) && rows16(a.dout, 2) &&
                   (reinterpret_cast<uintptr_t>(a.dq_accum) % 16 == 0);
  if (vec) {  // the kernel zeroes the dQ accumulator itself
    const dim3 grid((unsigned)((a.Tq_pad + kPreRows - 1) / kPreRows), (unsigned)(a.B * a.H));
    if (a.D == 128) preprocess_bf16_zero_kernel<128><<<grid, 256, 0, stream>>>(a);
    else preprocess_bf16_zero_kernel<64><<<grid, 256, 0, stream>>>(a);
    return cudaGetLastError();
  }
  // The dQ accumulator: B*H*Tq_pad*D floats (all of it in the padded layout of fa_bwd,
  // exactly [B*H, Tq, D] in the public preprocess entry point, where Tq_pad = Tq).
  cudaError_t e = cudaMemsetAsync(a.dq_accum, 0, (size_t)rows * a.D * sizeof(float), stream);
  if (e != cudaSuccess) return e;
  const unsigned grid = (unsigned)((rows + kRowsPerCta - 1) / kRowsPerCta);
  if (dtype == FA_DTYPE_F32) preprocess_kernel<float><<<grid, kRowsPerCta * 32, 0, stream>>>(a);
  else preprocess_kernel<__nv_bfloat16><<<grid, kRowsPerCta * 32, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_dq_convert(const AttnArgs& a, int dtype, cudaStream_t stream) {
  const int64_t rows = (int64_t)a.B * a.H * a.Tq;
  if (dtype == FA_DTYPE_BF16 && (a.D == 64 || a.D == 128) && rows16(a.dq, 2)) {
    const int64_t per_cta = 8LL * kVecPasses * (32 / (a.D / 4));
    const unsigned grid = (unsigned)((rows + per_cta - 1) / per_cta);
    if (a.D == 128) dq_convert_bf16_vec_kernel<128><<<grid, 256, 0, stream>>>(a);
    else dq_convert_bf16_vec_kernel<64><<<grid, 256, 0, stream>>>(a);
    return cudaGetLastError();
  }
  const unsigned grid = (unsigned)((rows + kRowsPerCta - 1) / kRowsPerCta);
  if (dtype == FA_DTYPE_F32) dq_convert_kernel<float><<<grid, kRowsPerCta * 32, 0, stream>>>(a);
  else dq_convert_kernel<__nv_bfloat16><<<grid, kRowsPerCta * 32, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_lse_merge(int rows, int D, float* o_acc, float* lse_acc, const void* o_part, int64_t stride,
                             int dtype, const float* lse_part, cudaStream_t stream) {
  const bool vec = dtype == FA_DTYPE_BF16 && (D == 64 || D == 128) && stride % 8 == 0 &&
                   (reinterpret_cast<uintptr_t>(o_part) & 15) == 0 && (reinterpret_cast<uintptr_t>(o_acc) & 15) == 0;
  if (vec) {
    const int per_cta = 8 * (32 / (D / 8)) * kMergePasses;
    const unsigned vgrid = (unsigned)((rows + per_cta - 1) / per_cta);
    const auto* op = static_cast<const __nv_bfloat16*>(o_part);
    if (D == 64)
      lse_merge_bf16_vec_kernel<64><<<vgrid, 256, 0, stream>>>(rows, o_acc, lse_acc, op, stride, lse_part);
    else
      lse_merge_bf16_vec_kernel<128><<<vgrid, 256, 0, stream>>>(rows, o_acc, lse_acc, op, stride, lse_part);
    return cudaGetLastError();
  }
  const unsigned grid = (unsigned)((rows + kRowsPerCta - 1) / kRowsPerCta);
  if (dtype == FA_DTYPE_F32)
    lse_merge_kernel<float><<<grid, kRowsPerCta * 32, 0, stream>>>(rows, D, o_acc, lse_acc,
                                                                   static_cast<const float*>(o_part), stride, lse_part);
  else
    lse_merge_kernel<__nv_bfloat16><<<grid, kRowsPerCta * 32, 0, stream>>>(
        rows, D, o_acc, lse_acc, static_cast<const __nv_bfloat16*>(o_part), stride, lse_part);
  return cudaGetLastError();
}

}  // namespace fa
