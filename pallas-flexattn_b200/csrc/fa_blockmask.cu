// GPU construction of FlexAttention block tables.  Tile coordinates are local; the
// mask sees global positions (q + q_offset, kv + kv_offset).
//
// classify_kernel replaces the host double loop of the reference's
// create_block_mask (src/pallas_flexattn/block_mask.py:54-129), which evaluates the
// mask on a 3x3 sample of each tile and synchronises with the host once per tile.
// Two rules are built:
//   REF9  the reference's rule, bit for bit: tile (i, j) is listed iff the mask is
//         true at any of q in {q0, (q0+q1)//2, q1-1} x kv in {k0, (k0+k1)//2, k1-1},
//         with q1 = min(q0 + block, Q_LEN), k1 = min(k0 + block, KV_LEN)
//         (block_mask.py:78-109).  Every listed tile is "partial".
//   EXACT tile listed iff any element is unmasked, and "full" (mask skipped in the
//         attention kernels) iff every element of the block_q x block_kv tile is
//         unmasked and inside KV_LEN.
// compact_rows / compact_cols turn the tile-class matrix into the kv_* row tables
// (sorted ascending, padded with -1 as block_mask.py:114-121 pads col_indices) and
// the transposed q_* tables the backward pass walks.
#include <cuda_runtime.h>

#include "fa_common.cuh"
#include "fa_internal.h"

namespace fa {
namespace {

constexpr int kClassifyThreads = 256;

__global__ void __launch_bounds__(kClassifyThreads)
    classify_kernel(const FaMaskSpec m, int Tq, int Tkv, int bq, int bkv, int mode, int nq, int nkv,
                    uint8_t* tile_class) {
  const int kb = blockIdx.x, qb = blockIdx.y, bb = blockIdx.z;
  const MaskCtx mc = make_mask_ctx(m, bb, Tkv);
  const int q0 = qb * bq, q1 = min(q0 + bq, Tq);
  const int k0 = kb * bkv, k1 = min(k0 + bkv, Tkv);
  uint8_t cls;
  if (mode == FA_BLOCK_MASK_REF9) {
    bool v = false;
    if (threadIdx.x < 9) {
      const int qs[3] = {q0, (q0 + q1) / 2, q1 - 1};
      const int ks[3] = {k0, (k0 + k1) / 2, k1 - 1};
      const int q = qs[threadIdx.x / 3], kv = ks[threadIdx.x % 3];
      const int dq = (mc.flags & FA_MASK_DOCUMENT) ? mc.doc_q[q + mc.q_off] : 0;
      v = mask_ok(mc, q + mc.q_off, kv + mc.kv_off, dq);
    }
    cls = __syncthreads_or(v) ? 1 : 0;
  } else {
    // Evaluate the whole block_q x block_kv tile (columns past KV_LEN count as masked).
    const int rows = q1 - q0;
    const int64_t n = (int64_t)rows * bkv;
    bool any = false, all = true;
    for (int64_t base = 0; base < n; base += 8 * kClassifyThreads) {
      for (int64_t u = 0; u < 8; ++u) {
        const int64_t idx = base + u * kClassifyThreads + threadIdx.x;
        if (idx >= n) break;
        const int q = q0 + (int)(idx / bkv), kv = k0 + (int)(idx % bkv);
        const int dq = (mc.flags & FA_MASK_DOCUMENT) ? mc.doc_q[q + mc.q_off] : 0;
        const bool v = mask_ok(mc, q + mc.q_off, kv + mc.kv_off, dq);
        any = any || v;
        all = all && v;
      }
      const bool a_any = __syncthreads_or(any);
      const bool a_all = __syncthreads_and(all);
      any = a_any;
      all = a_all;
      if (any && !all) break;  // already known to be partial
    }
    cls = any ? (all ? 2 : 1) : 0;
  }
  if (threadIdx.x == 0) tile_class[((int64_t)bb * nq + qb) * nkv + kb] = cls;
}

// One warp per (batch, q block): list partial and full kv blocks in ascending order.
__global__ void compact_rows_kernel(const uint8_t* tile_class, int num_b, int nq, int nkv, int32_t* kv_num,
                                    int32_t* kv_idx, int32_t* full_num, int32_t* full_idx) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= num_b * nq) return;
  const uint8_t* cls = tile_class + (int64_t)warp * nkv;
  int32_t* pi = kv_idx + (int64_t)warp * nkv;
  int32_t* fi = full_idx + (int64_t)warp * nkv;
  int np = 0, nf = 0;
  for (int j0 = 0; j0 < nkv; j0 += 32) {
    const int j = j0 + lane;
    int c = j < nkv ? cls[j] : 0;
    if (c == 3) c = 1;
    const unsigned mp = __ballot_sync(0xffffffffu, c == 1);
    const unsigned mf = __ballot_sync(0xffffffffu, c == 2);
    const unsigned below = (1u << lane) - 1u;
    if (c == 1) pi[np + __popc(mp & below)] = j;
    if (c == 2) fi[nf + __popc(mf & below)] = j;
    np += __popc(mp);
    nf += __popc(mf);
  }
  for (int e = np + lane; e < nkv; e += 32) pi[e] = -1;
  for (int e = nf + lane; e < nkv; e += 32) fi[e] = -1;
  if (lane == 0) {
    kv_num[warp] = np;
    full_num[warp] = nf;
  }
}

// One warp per (batch, kv block): the transposed lists.
__global__ void compact_cols_kernel(const uint8_t* tile_class, int num_b, int nq, int nkv, int32_t* q_num,
                                    int32_t* q_idx, int32_t* full_num, int32_t* full_idx) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= num_b * nkv) return;
  const int bb = warp / nkv, kb = warp % nkv;
  const uint8_t* cls = tile_class + (int64_t)bb * nq * nkv + kb;
  int32_t* pi = q_idx + (int64_t)warp * nq;
  int32_t* fi = full_idx + (int64_t)warp * nq;
  int np = 0, nf = 0;
  for (int i0 = 0; i0 < nq; i0 += 32) {
    const int i = i0 + lane;
    int c = i < nq ? cls[(int64_t)i * nkv] : 0;
    if (c == 3) c = 1;
    const unsigned mp = __ballot_sync(0xffffffffu, c == 1);
    const unsigned mf = __ballot_sync(0xffffffffu, c == 2);
    const unsigned below = (1u << lane) - 1u;
    if (c == 1) pi[np + __popc(mp & below)] = i;
    if (c == 2) fi[nf + __popc(mf & below)] = i;
    np += __popc(mp);
    nf += __popc(mf);
  }
  for (int e = np + lane; e < nq; e += 32) pi[e] = -1;
  for (int e = nf + lane; e < nq; e += 32) fi[e] = -1;
  if (lane == 0) {
    q_num[warp] = np;
    full_num[warp] = nf;
  }
}

// Scatter row lists into the tile-class matrix (1 partial, 2 full, 3 both).
__global__ void scatter_lists_kernel(int rows, int nkv, int cap, const int32_t* num, const int32_t* idx, int code,
                                     uint8_t* tile_class) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (int64_t)rows * cap) return;
  const int row = (int)(t / cap), e = (int)(t % cap);
  if (e >= num[row]) return;
  const int j = idx[(int64_t)row * cap + e];
  if (j < 0 || j >= nkv) return;
  tile_class[(int64_t)row * nkv + j] |= (uint8_t)code;  // a tile is listed at most once per list
}

cudaError_t compact_all(const FaBlockMaskOut& out, cudaStream_t stream) {
  const int threads = 256, wpb = threads / 32;
  const int rows = out.num_b * out.nq, cols = out.num_b * out.nkv;
  compact_rows_kernel<<<(rows + wpb - 1) / wpb, threads, 0, stream>>>(out.tile_class, out.num_b, out.nq, out.nkv,
                                                                       out.kv_num_blocks, out.kv_indices,
                                                                       out.full_kv_num_blocks, out.full_kv_indices);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  compact_cols_kernel<<<(cols + wpb - 1) / wpb, threads, 0, stream>>>(out.tile_class, out.num_b, out.nq, out.nkv,
                                                                       out.q_num_blocks, out.q_indices,
                                                                       out.full_q_num_blocks, out.full_q_indices);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_create_block_mask(const FaMaskSpec& m, int B, int Tq, int Tkv, int bq, int bkv, int mode,
                                     const FaBlockMaskOut& out, cudaStream_t stream) {
  (void)B;
  const dim3 grid((unsigned)out.nkv, (unsigned)out.nq, (unsigned)out.num_b);
  classify_kernel<<<grid, kClassifyThreads, 0, stream>>>(m, Tq, Tkv, bq, bkv, mode, out.nq, out.nkv, out.tile_class);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return compact_all(out, stream);
}

cudaError_t launch_tables_from_lists(int num_b, int nq, int nkv, const int32_t* kv_num, const int32_t* kv_idx,
                                     const int32_t* full_num, const int32_t* full_idx, int kv_cap,
                                     const FaBlockMaskOut& out, cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(out.tile_class, 0, (size_t)num_b * nq * nkv, stream);
  if (e != cudaSuccess) return e;
  const int rows = num_b * nq;
  const int64_t n = (int64_t)rows * kv_cap;
  const unsigned grid = (unsigned)((n + 255) / 256);
  if (kv_num) {
    scatter_lists_kernel<<<grid, 256, 0, stream>>>(rows, nkv, kv_cap, kv_num, kv_idx, 1, out.tile_class);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (full_num) {
    scatter_lists_kernel<<<grid, 256, 0, stream>>>(rows, nkv, kv_cap, full_num, full_idx, 2, out.tile_class);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  return compact_all(out, stream);
}

}  // namespace fa
