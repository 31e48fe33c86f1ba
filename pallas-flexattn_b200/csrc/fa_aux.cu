// HBM-bound helper kernels of the backward pass and the context-parallel ring.
//
//   bwd_preprocess  delta = rowsum(O * dO) in fp32 (reference:
//                   flash_attention_bwd_preprocess_kernel, src/pallas_flexattn/
//                   flash_attn.py:168-173, which stores it in O's dtype) and zeroes
//                   the fp32 dQ accumulator in the same pass.
//   dq_convert      dQ = scale * dq_accum, cast to the input dtype.
//   lse_merge       combine two partial (O, logsumexp) results over disjoint keys.
// One warp per row; each lane moves 16-byte vectors where alignment allows.
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

// Zeroes D floats of the dQ accumulator per padded row, B*H*Tq_pad*D in all (the
// [B*H, Tq, D] accumulator is the first B*H*Tq*D of them).
__device__ __forceinline__ void zero_dq_row(const AttnArgs& a, int64_t prow, int lane) {
  float4* z = reinterpret_cast<float4*>(a.dq_accum + prow * a.D);
  for (int d4 = lane; d4 < a.D / 4; d4 += 32) z[d4] = make_float4(0.f, 0.f, 0.f, 0.f);
}

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
    zero_dq_row(a, prow, lane);
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
  zero_dq_row(a, prow, lane);
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

}  // namespace

cudaError_t launch_bwd_preprocess(const AttnArgs& a, int dtype, cudaStream_t stream) {
  const int64_t rows = (int64_t)a.B * a.H * a.Tq_pad;
  const unsigned grid = (unsigned)((rows + kRowsPerCta - 1) / kRowsPerCta);
  if (dtype == FA_DTYPE_F32) preprocess_kernel<float><<<grid, kRowsPerCta * 32, 0, stream>>>(a);
  else preprocess_kernel<__nv_bfloat16><<<grid, kRowsPerCta * 32, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_dq_convert(const AttnArgs& a, int dtype, cudaStream_t stream) {
  const int64_t rows = (int64_t)a.B * a.H * a.Tq;
  const unsigned grid = (unsigned)((rows + kRowsPerCta - 1) / kRowsPerCta);
  if (dtype == FA_DTYPE_F32) dq_convert_kernel<float><<<grid, kRowsPerCta * 32, 0, stream>>>(a);
  else dq_convert_kernel<__nv_bfloat16><<<grid, kRowsPerCta * 32, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_lse_merge(int rows, int D, float* o_acc, float* lse_acc, const void* o_part, int64_t stride,
                             int dtype, const float* lse_part, cudaStream_t stream) {
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
