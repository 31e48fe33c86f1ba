// FlexAttention backward for B200 (sm_100a): TMA + tcgen05 + TMEM, warp-specialised.
//
// Replaces the reference's two backward kernels (src/pallas_flexattn/flash_attn.py:
// dK/dV :206-253 and dQ :313-356), which recompute S and P twice (7 tile GEMMs per
// tile pair), with one KV-stationary kernel doing 5:
//   St  = K Q_i^T          dPt = V dO_i^T          (TMEM, fp32)
//   Pt  = exp2(score(St) - lse2_i)   dSt = Pt * (dPt - delta_i) * score'   (registers)
//   dV += Pt dO_i  (A = Pt from TMEM)   dK += dSt Q_i   dQ_i = dS K   (fp32 in TMEM)
// dQ_i is added into an fp32 accumulator in global memory with TMA reduce-add by a
// dedicated warpgroup; fa_bwd scales and converts it afterwards.  The CTA walks the
// transposed block table (q_indices / full_q_indices) of its kv tile, skipping empty
// tiles; full tiles do not evaluate the mask.
//
// Warp roles (512 threads, four warpgroups):
//   WG0, WG1 (warps 0-7)  compute: thread = kv row; WG0 takes q columns 0-63, WG1 64-127
//   WG2 (warps 8-11)      dQ drain: thread = q row; TMEM -> swizzled smem -> TMA reduce-add
//   WG3 (warps 12-15)     warp 12 TMA producer, warp 13 MMA issuer + TMEM owner, 14-15 idle
// Registers: launched at 128 per thread (512 x 128 = 65536); setmaxnreg moves them to
// 176 for WG0/WG1, 80 for WG2, 80 for WG3 (2*128*176 + 128*80 + 128*80 = 65536).
// TMEM columns: St [0,128) (Pt bf16 written back into its own half), dPt [128,256)
// (reused for dQ_i once dSt is in shared memory), dV [256,256+D), dK [256+D,256+2D).
// dSt is stored once in shared memory in the 128-byte-swizzled K-major layout; the
// dK MMA reads it as K-major (M = kv) and the dQ MMA as MN-major (M = q).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "fa_common.cuh"
#include "fa_internal.h"
#include "fa_ptx.cuh"

namespace fa {

namespace {

constexpr int kBM = 128;  // kv rows per CTA
constexpr int kBQ = 128;  // q rows per iteration
constexpr int kBwdThreads = 512;
constexpr int kWarpDq0 = 8, kWarpProd = 12, kWarpMma = 13;
constexpr int kRegsCompute = 176, kRegsDrain = 80, kRegsCtl = 80;
constexpr int kChunk = 128 * 64 * 2;  // one 64-column swizzle panel of a 128-row bf16 tile
constexpr int kDqStage = 32 * 32 * 4;  // per drain warp: 32 rows x 32 fp32, 128B-swizzled

struct BwdSmemLayout {
  int tile, nq_st, no_st, k_off, v_off, q_off, o_off, ds_off, dq_off, lse_off, dl_off, bar_off, misc_off, cls_off,
      ent_off, total;
};

__host__ __device__ inline BwdSmemLayout bwd_smem_layout(int D, int nq_st, int no_st, int nq) {
  BwdSmemLayout L;
  L.tile = kBM * D * 2;
  L.nq_st = nq_st;
  L.no_st = no_st;
  L.k_off = 0;
  L.v_off = L.tile;
  L.q_off = 2 * L.tile;
  L.o_off = L.q_off + nq_st * L.tile;
  L.ds_off = L.o_off + no_st * L.tile;
  L.dq_off = L.ds_off + kBQ * kBM * 2;
  L.lse_off = L.dq_off + 4 * kDqStage;
  L.dl_off = L.lse_off + nq_st * kBQ * 4;
  L.bar_off = L.dl_off + nq_st * kBQ * 4;
  L.misc_off = L.bar_off + (2 * nq_st + 2 * no_st + 12) * 8;
  L.cls_off = L.misc_off + 16;
  L.ent_off = L.cls_off + 4 * nq;
  L.total = L.ent_off + 4 * nq + 1024;
  return L;
}

template <int D, int SK>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                  const __grid_constant__ CUtensorMap tm_dq, const AttnArgs a, const int NQS, const int NOS) {
  constexpr int NCHUNK = D / 64;
  constexpr uint32_t TM_S = 0, TM_DP = 128, TM_DV = 256, TM_DK = 256 + D;
  constexpr uint32_t IDESC_SQ = make_idesc_bf16(kBM, kBQ, 0, 0);  // St, dPt: N = q
  constexpr uint32_t IDESC_KV = make_idesc_bf16(kBM, D, 0, 1);    // dV, dK: A K-major, B MN-major
  constexpr uint32_t IDESC_DQ = make_idesc_bf16(kBQ, D, 1, 1);    // dQ: A, B MN-major

  const int nq = a.bt.nq;
  const BwdSmemLayout L = bwd_smem_layout(D, NQS, NOS, nq);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem + L.k_off;
  uint8_t* sV = smem + L.v_off;
  uint8_t* sQ = smem + L.q_off;
  uint8_t* sO = smem + L.o_off;
  uint8_t* sdS = smem + L.ds_off;
  uint8_t* sDq = smem + L.dq_off;
  float* sLse = reinterpret_cast<float*>(smem + L.lse_off);
  float* sDl = reinterpret_cast<float*>(smem + L.dl_off);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* bar_kv = bars;
  uint64_t* bar_q_full = bars + 1;
  uint64_t* bar_q_empty = bar_q_full + NQS;
  uint64_t* bar_o_full = bar_q_empty + NQS;
  uint64_t* bar_o_empty = bar_o_full + NOS;
  uint64_t* bar_s_full = bar_o_empty + NOS;
  uint64_t* bar_dp_full = bar_s_full + 1;
  uint64_t* bar_p_full = bar_s_full + 2;
  uint64_t* bar_ds_full = bar_s_full + 3;
  uint64_t* bar_ds_empty = bar_s_full + 4;
  uint64_t* bar_dq_full = bar_s_full + 5;
  uint64_t* bar_dq_empty = bar_s_full + 6;
  uint64_t* bar_dkv_full = bar_s_full + 7;
  uint64_t* bar_teardown = bar_s_full + 8;
  int* misc = reinterpret_cast<int*>(smem + L.misc_off);
  volatile int* abort_flag = misc;
  int* n_entries_s = misc + 1;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(misc + 2);
  int* cls = reinterpret_cast<int*>(smem + L.cls_off);
  int* entries = reinterpret_cast<int*>(smem + L.ent_off);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int BH = a.B * a.H;
  const int bh = blockIdx.x % BH;
  const int j = blockIdx.x / BH;  // kv tile; low j first (the most q tiles under causal masks)
  const int b = bh / a.H, h = bh % a.H;
  const int Tq_pad = (a.Tq + kBQ - 1) / kBQ * kBQ;

  if (warp == kWarpProd && lane == 0) {
    mbar_init(bar_kv, 1);
    for (int s = 0; s < NQS; ++s) {
      mbar_init(bar_q_full + s, 1);
      mbar_init(bar_q_empty + s, 1);
    }
    for (int s = 0; s < NOS; ++s) {
      mbar_init(bar_o_full + s, 1);
      mbar_init(bar_o_empty + s, 1);
    }
    mbar_init(bar_s_full, 1);
    mbar_init(bar_dp_full, 1);
    mbar_init(bar_p_full, 256);
    mbar_init(bar_ds_full, 256);
    mbar_init(bar_ds_empty, 1);
    mbar_init(bar_dq_full, 1);
    mbar_init(bar_dq_empty, 128);
    mbar_init(bar_dkv_full, 1);
    mbar_init(bar_teardown, 1);
    misc[0] = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_dq);
  }
  if (warp == kWarpMma) {
    tmem_alloc(tmem_base_s, 512);
    tmem_relinquish();
  }
  for (int i = tid; i < nq; i += kBwdThreads) cls[i] = 0;
  __syncthreads();
  {
    const int64_t row = table_head(a.bt, b, h) * a.bt.nkv + j;
    const int np = a.bt.q_num_blocks ? a.bt.q_num_blocks[row] : 0;
    for (int e = tid; e < np; e += kBwdThreads) {
      const int i = a.bt.q_indices[row * a.bt.q_cap + e];
      if (i >= 0 && i < nq) atomicOr(&cls[i], 1);
    }
    const int nf = a.bt.full_q_num_blocks ? a.bt.full_q_num_blocks[row] : 0;
    for (int e = tid; e < nf; e += kBwdThreads) {
      const int i = a.bt.full_q_indices[row * a.bt.q_cap + e];
      if (i >= 0 && i < nq) atomicOr(&cls[i], 2);
    }
  }
  __syncthreads();
  if (warp == kWarpProd) {
    int base = 0;
    for (int i0 = 0; i0 < nq; i0 += 32) {
      const int i = i0 + lane;
      int c = (i < nq) ? cls[i] : 0;
      if (c == 3) c = 1;
      const unsigned m = __ballot_sync(0xffffffffu, c != 0);
      if (c) entries[base + __popc(m & ((1u << lane) - 1u))] = i | (c << 24);
      base += __popc(m);
    }
    if (lane == 0) *n_entries_s = base;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_s;
  const int n_ent = *n_entries_s;

  if (warp >= kWarpProd) {
    setmaxnreg_dec<kRegsCtl>();
    if (warp == kWarpProd) {
      // ---------------------------------------------------------------- TMA producer
      if (lane == 0 && n_ent > 0) {
        mbar_arrive_expect_tx(bar_kv, 2 * L.tile);
        for (int c = 0; c < NCHUNK; ++c) {
          tma_load_4d(sK + c * kChunk, &tm_k, bar_kv, c * 64, j * kBM, h, b);
          tma_load_4d(sV + c * kChunk, &tm_v, bar_kv, c * 64, j * kBM, h, b);
        }
        const float* lse2 = a.lse2 + (int64_t)bh * Tq_pad;
        const float* dl = a.delta + (int64_t)bh * Tq_pad;
        bool ok = true;
        int issued_q = 0, issued_o = 0;
        for (int t = 0; t < n_ent && ok; ++t) {
          const int i = entries[t] & 0xFFFFFF;
          const int qs = t % NQS, qu = t / NQS;
          if (!mbar_wait(bar_q_empty + qs, (qu & 1) ^ 1, abort_flag)) { ok = false; break; }
          // lse2 and delta ride with Q: the Q slot is released only after dSt is built, which
          // is the last read of both (the dO slot is released earlier, after the dV MMA).
          mbar_arrive_expect_tx(bar_q_full + qs, L.tile + 2 * kBQ * 4);
          for (int c = 0; c < NCHUNK; ++c)
            tma_load_4d(sQ + qs * L.tile + c * kChunk, &tm_q, bar_q_full + qs, c * 64, i * kBQ, h, b);
          bulk_load(sLse + qs * kBQ, lse2 + i * kBQ, kBQ * 4, bar_q_full + qs);
          bulk_load(sDl + qs * kBQ, dl + i * kBQ, kBQ * 4, bar_q_full + qs);
          ++issued_q;
          const int os = t % NOS, ou = t / NOS;
          if (!mbar_wait(bar_o_empty + os, (ou & 1) ^ 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(bar_o_full + os, L.tile);
          for (int c = 0; c < NCHUNK; ++c)
            tma_load_4d(sO + os * L.tile + c * kChunk, &tm_do, bar_o_full + os, c * 64, i * kBQ, h, b);
          ++issued_o;
        }
        if (!ok) {
          report_status(a.status, FA_ERR_TIMEOUT);
          *abort_flag = 1;
        }
        // Teardown: no bulk copy may still be writing this CTA's shared memory.
        volatile int never = 0;
        mbar_wait(bar_kv, 0, &never);
        for (int s = 0; s < NQS && s < issued_q; ++s) {
          const int last = s + ((issued_q - 1 - s) / NQS) * NQS;
          mbar_wait(bar_q_full + s, (last / NQS) & 1, &never);
        }
        for (int s = 0; s < NOS && s < issued_o; ++s) {
          const int last = s + ((issued_o - 1 - s) / NOS) * NOS;
          mbar_wait(bar_o_full + s, (last / NOS) & 1, &never);
        }
      }
    } else if (warp == kWarpMma) {
      // ---------------------------------------------------------------- MMA issuer
      if (lane == 0 && n_ent > 0) {
        // Descriptors are built once; per K step only the start-address field of the low
        // word moves (see mma_ss_lh).  K-major: LBO 16 B; MN-major: LBO = one 64-column
        // panel; SBO = 1024 B for both.  kofs/mofs are the per-step offsets in 16-byte units.
        const uint64_t d0 = make_smem_desc(smem_u32(sK), 16, 1024, SMEM_SWIZZLE_128B);
        const uint32_t hi = (uint32_t)(d0 >> 32);
        const uint32_t kmaj = (uint32_t)d0 - ((smem_u32(sK) >> 4) & 0x3FFFu);  // LBO bits only
        const uint32_t mnmaj = (uint32_t)make_smem_desc(0, kChunk, 1024, SMEM_SWIZZLE_128B);
        auto lo = [](uint32_t lbo_bits, const void* p) { return lbo_bits + ((smem_u32(p) >> 4) & 0x3FFFu); };
        const uint32_t K_k = lo(kmaj, sK), K_mn = lo(mnmaj, sK), V_k = lo(kmaj, sV), S_k = lo(kmaj, sdS),
                       S_mn = lo(mnmaj, sdS);
        const uint32_t Q_k0 = lo(kmaj, sQ), Q_mn0 = lo(mnmaj, sQ), O_k0 = lo(kmaj, sO), O_mn0 = lo(mnmaj, sO);
        const uint32_t tile16 = (uint32_t)L.tile >> 4;
        auto kofs = [](int kk) { return (uint32_t)((kk >> 2) * (kChunk >> 4) + (kk & 3) * 2); };
        auto mofs = [](int kk) { return (uint32_t)(kk * (2048 >> 4)); };
        bool ok = mbar_wait(bar_kv, 0, abort_flag);
        tc_fence_after();
        for (int t = 0; t < n_ent && ok; ++t) {
          const int qs = t % NQS, os = t % NOS;
          const uint32_t ph = t & 1;
          const uint32_t Q_k = Q_k0 + qs * tile16, Q_mn = Q_mn0 + qs * tile16;
          const uint32_t O_k = O_k0 + os * tile16, O_mn = O_mn0 + os * tile16;
          const uint32_t acc0 = t > 0 ? 1u : 0u;
          // St = K Q^T
          if (!(ok = mbar_wait(bar_q_full + qs, (t / NQS) & 1, abort_flag))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_ss_lh(tmem_base + TM_S, K_k + kofs(kk), hi, Q_k + kofs(kk), hi, IDESC_SQ, kk > 0);
          tc_commit(bar_s_full);
          // dPt = V dO^T (its columns also hold dQ of the previous step until drained)
          if (!(ok = mbar_wait(bar_o_full + os, (t / NOS) & 1, abort_flag))) break;
          if (t > 0 && !(ok = mbar_wait(bar_dq_empty, ph ^ 1, abort_flag))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_ss_lh(tmem_base + TM_DP, V_k + kofs(kk), hi, O_k + kofs(kk), hi, IDESC_SQ, kk > 0);
          tc_commit(bar_dp_full);
          // dV += Pt dO  (Pt of q columns 0-63 at St cols 0-31, 64-127 at cols 64-95)
          if (!(ok = mbar_wait(bar_p_full, ph, abort_flag))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kBQ / 16; ++kk)
            mma_ts_lh(tmem_base + TM_DV, tmem_base + TM_S + (kk < 4 ? kk * 8 : 64 + (kk - 4) * 8), O_mn + mofs(kk),
                      hi, IDESC_KV, kk > 0 ? 1u : acc0);
          tc_commit(bar_o_empty + os);
          // dK += dSt Q ; dQ_i = dS K
          if (!(ok = mbar_wait(bar_ds_full, ph, abort_flag))) break;
          tc_fence_after();
          // dQ first: the drain (and, through it, the next dPt) waits on it; dK runs meanwhile.
#pragma unroll
          for (int kk = 0; kk < kBM / 16; ++kk)
            mma_ss_lh(tmem_base + TM_DP, S_mn + mofs(kk), hi, K_mn + mofs(kk), hi, IDESC_DQ, kk > 0);
          tc_commit(bar_dq_full);
#pragma unroll
          for (int kk = 0; kk < kBQ / 16; ++kk)
            mma_ss_lh(tmem_base + TM_DK, S_k + kofs(kk), hi, Q_mn + mofs(kk), hi, IDESC_KV, kk > 0 ? 1u : acc0);
          tc_commit(bar_q_empty + qs);
          tc_commit(bar_ds_empty);
        }
        if (ok) tc_commit(bar_dkv_full);
        if (!ok) {
          report_status(a.status, FA_ERR_TIMEOUT);
          *abort_flag = 1;
        }
        tc_commit(bar_teardown);
        volatile int never = 0;
        mbar_wait(bar_teardown, 0, &never);
      }
      __syncwarp();
    }
  } else if (warp >= kWarpDq0) {
    setmaxnreg_dec<kRegsDrain>();
    // ------------------------------------------------------------------ dQ drain (thread = q row)
    const int wq = warp & 3;
    const uint32_t t_dq = tmem_base + ((uint32_t)(wq * 32) << 16) + TM_DP;
    uint8_t* stage = sDq + wq * kDqStage;
    bool ok = true;
    for (int t = 0; t < n_ent && ok; ++t) {
      const int i = entries[t] & 0xFFFFFF;
      if (!(ok = mbar_wait(bar_dq_full, t & 1, abort_flag))) break;
      tc_fence_after();
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(t_dq + c0, v);
        tmem_ld_wait();
        reg_pin(v);
        if (c0 + 32 == D) {  // all of dQ_i is in registers: its TMEM columns may be reused
          tc_fence_before();
          mbar_arrive(bar_dq_empty);
        }
        if (lane == 0) bulk_wait_read_all();  // the previous reduce has read the stage
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 8; ++u)
          *reinterpret_cast<uint4*>(stage + lane * 128 + ((u ^ (lane & 7)) << 4)) =
              make_uint4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_3d(&tm_dq, stage, c0, i * kBQ + wq * 32, bh);
          bulk_commit_group();
        }
      }
    }
    if (lane == 0) bulk_wait_all();
    if (!ok) {
      report_status(a.status, FA_ERR_TIMEOUT);
      *abort_flag = 1;
    }
  } else {
    setmaxnreg_inc<kRegsCompute>();
    // ------------------------------------------------------------------ compute (thread = kv row)
    const int wg = warp >> 2;
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const int kv = j * kBM + r;
    const int cbase = wg * 64;
    const uint32_t t_lane = tmem_base + ((uint32_t)(wq * 32) << 16);
    const ScoreCtx sc = make_score_ctx(a.score, a.scale, h, a.Tkv);
    const MaskCtx mc = make_mask_ctx(a.mask, b, a.Tkv);
    const int kvg = kv + mc.kv_off;
    const float inv_cap_log2 = sc.inv_cap * kLn2;  // 1 / (cap * log2(e))
    // Causal, window and the Tq/Tkv bounds intersect to one allowed q interval [q_lo, q_hi]
    // (global positions) for this thread's kv row; partial tiles test it with two compares.
    // Document and tile-table predicates, when enabled, are evaluated per element on top.
    int q_lo = mc.q_off, q_hi = mc.q_off + a.Tq - 1;
    if (kvg >= mc.Tkv) q_hi = q_lo - 1;
    if (mc.flags & FA_MASK_CAUSAL) q_lo = max(q_lo, kvg);
    if (mc.flags & FA_MASK_WINDOW) {
      if (mc.left >= 0) q_hi = min(q_hi, kvg + mc.left);
      if (mc.right >= 0) q_lo = max(q_lo, kvg - mc.right);
    }
    const bool per_elem_mask = (mc.flags & (FA_MASK_DOCUMENT | FA_MASK_TILE_TABLE)) != 0;
    bool ok = true;
    for (int t = 0; t < n_ent && ok; ++t) {
      const int e = entries[t];
      const int i = e & 0xFFFFFF;
      const bool partial = ((e >> 24) & 3) == 1;
      const int qs = t % NQS;
      const uint32_t ph = t & 1;
      const float* lse2 = sLse + qs * kBQ + cbase;
      const float* dl = sDl + qs * kBQ + cbase;
      const int q0 = i * kBQ + cbase;

      if (!(ok = mbar_wait(bar_s_full, ph, abort_flag))) break;
      tc_fence_after();
      // p stays fp32 until dSt is formed; each 32-column half of Pt goes back to TMEM (bf16,
      // into already-read S columns) as soon as it is computed, to keep registers low.
      float p[64];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t s[32];
        tmem_ld32(t_lane + TM_S + cbase + 32 * hh, s);
        float l2[32];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float4 v4 = reinterpret_cast<const float4*>(lse2 + 32 * hh)[u];
          l2[4 * u] = v4.x; l2[4 * u + 1] = v4.y; l2[4 * u + 2] = v4.z; l2[4 * u + 3] = v4.w;
        }
        tmem_ld_wait();
        reg_pin(s);
        const int qg0 = q0 + 32 * hh + mc.q_off;  // global position of column 0 of this half
#pragma unroll
        for (int c = 0; c < 32; ++c)
          p[32 * hh + c] = ex2_approx(score_log2<SK>(__uint_as_float(s[c]), qg0 + c, kvg, sc) - l2[c]);
        if (partial) {
          const unsigned span = (unsigned)(q_hi - q_lo);
          const int clo = q_lo - qg0;
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if ((unsigned)(c - clo) > span || q_hi < q_lo) p[32 * hh + c] = 0.f;
          if (per_elem_mask) {
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const int q = qg0 - mc.q_off + c;  // local row
              const int dq = (mc.flags & FA_MASK_DOCUMENT) && q < a.Tq ? __ldg(mc.doc_q + qg0 + c) : 0;
              if (!mask_ok(mc, qg0 + c, kvg, dq)) p[32 * hh + c] = 0.f;
            }
          }
        }
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) pk[c] = pack_bf16x2(p[32 * hh + 2 * c], p[32 * hh + 2 * c + 1]);
        tmem_st16(t_lane + TM_S + (wg ? 64 : 0) + 16 * hh, pk);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar_p_full);

      if (!(ok = mbar_wait(bar_dp_full, ph, abort_flag))) break;
      if (t > 0 && !(ok = mbar_wait(bar_ds_empty, ph ^ 1, abort_flag))) break;
      tc_fence_after();
      uint8_t* ds_row = sdS + wg * kChunk + r * 128;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t dp[32];
        tmem_ld32(t_lane + TM_DP + cbase + 32 * hh, dp);
        float dl32[32];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float4 v4 = reinterpret_cast<const float4*>(dl + 32 * hh)[u];
          dl32[4 * u] = v4.x; dl32[4 * u + 1] = v4.y; dl32[4 * u + 2] = v4.z; dl32[4 * u + 3] = v4.w;
        }
        tmem_ld_wait();
        reg_pin(dp);
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const int cc = 32 * hh + c;
          float d0 = p[cc] * (__uint_as_float(dp[c]) - dl32[c]);
          float d1 = p[cc + 1] * (__uint_as_float(dp[c + 1]) - dl32[c + 1]);
          if constexpr (SK == SC_SOFTCAP || SK == SC_GENERAL) {
            // Softcap derivative 1 - t^2, with t = x / cap_log2 recovered from p = 2^(x - lse2)
            // instead of being held in registers since the P phase.  p = 0 means dS = 0.
            if (sc.flags & FA_SCORE_SOFTCAP) {
              const float x0 = lg2_approx(p[cc]) + lse2[cc], x1 = lg2_approx(p[cc + 1]) + lse2[cc + 1];
              const float t0 = x0 * inv_cap_log2, t1 = x1 * inv_cap_log2;
              d0 *= p[cc] > 0.f ? fmaf(-t0, t0, 1.f) : 1.f;
              d1 *= p[cc + 1] > 0.f ? fmaf(-t1, t1, 1.f) : 1.f;
            }
          }
          pk[c >> 1] = pack_bf16x2(d0, d1);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int unit = 4 * hh + u;  // 16-byte unit within the 128-byte row
          *reinterpret_cast<uint4*>(ds_row + ((unit ^ (r & 7)) << 4)) =
              make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar_ds_full);
    }
    if (!ok) {
      report_status(a.status, FA_ERR_TIMEOUT);
      *abort_flag = 1;
    }
    // ------------------------------------------------------------------ epilogue: dK, dV rows
    bool have = ok && n_ent > 0;
    if (have) {
      have = mbar_wait(bar_dkv_full, 0, abort_flag);
      if (!have) {
        report_status(a.status, FA_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      tc_fence_after();
    }
    __nv_bfloat16* dvr = reinterpret_cast<__nv_bfloat16*>(a.dv.ptr) + (int64_t)b * a.dv.stride_b +
                         (int64_t)h * a.dv.stride_h + (int64_t)kv * a.dv.stride_t;
    __nv_bfloat16* dkr = reinterpret_cast<__nv_bfloat16*>(a.dk.ptr) + (int64_t)b * a.dk.stride_b +
                         (int64_t)h * a.dk.stride_h + (int64_t)kv * a.dk.stride_t;
#pragma unroll 1
    for (int which = 0; which < 2; ++which) {
      const float mul = which ? a.scale : 1.f;
      __nv_bfloat16* dst = which ? dkr : dvr;
      const uint32_t tcol = which ? TM_DK : TM_DV;
#pragma unroll 1
      for (int c0 = wg * (D / 2); c0 < (wg + 1) * (D / 2); c0 += 32) {
        uint32_t v[32];
        if (have) {
          tmem_ld32(t_lane + tcol + c0, v);
          tmem_ld_wait();
          reg_pin(v);
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = 0u;
        }
        if (kv < a.Tkv) {
          uint32_t pk[16];
#pragma unroll
          for (int c = 0; c < 32; c += 2)
            pk[c >> 1] = pack_bf16x2(__uint_as_float(v[c]) * mul, __uint_as_float(v[c + 1]) * mul);
          uint4* d4 = reinterpret_cast<uint4*>(dst + c0);
#pragma unroll
          for (int u = 0; u < 4; ++u) d4[u] = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
      }
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

bool pick_stages(int D, int nq, int* nqs, int* nos) {
  const int cand[4][2] = {{2, 2}, {2, 1}, {1, 1}, {0, 0}};
  for (int c = 0; cand[c][0]; ++c)
    if (bwd_smem_layout(D, cand[c][0], cand[c][1], nq).total <= 227 * 1024) {
      *nqs = cand[c][0];
      *nos = cand[c][1];
      return true;
    }
  return false;
}

}  // namespace

int bwd_tc_max_stages(int D, int nq) {
  int a = 0, b = 0;
  return pick_stages(D, nq, &a, &b) ? a : 0;
}

cudaError_t launch_bwd_tc(const AttnArgs& a, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                          const CUtensorMap& tdo, const CUtensorMap& tdq, cudaStream_t stream) {
  int nqs = 0, nos = 0;
  if (!pick_stages(a.D, a.bt.nq, &nqs, &nos)) return cudaErrorInvalidValue;
  if (a.num_stages > 0 && a.num_stages < nqs) nqs = a.num_stages;
  const int smem = bwd_smem_layout(a.D, nqs, nos, a.bt.nq).total;
  const dim3 grid((unsigned)(a.bt.nkv * a.B * a.H));
  const int sk = score_kind_of(a.score.flags);
  auto go = [&](auto kern) -> cudaError_t {
    // The register split must fit the launch allocation, or setmaxnreg.inc would wait forever.
    cudaFuncAttributes fa_attr;
    cudaError_t e = cudaFuncGetAttributes(&fa_attr, kern);
    if (e != cudaSuccess) return e;
    if (fa_attr.numRegs * kBwdThreads < 2 * 128 * kRegsCompute + 128 * kRegsDrain + 128 * kRegsCtl)
      return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, kBwdThreads, smem, stream>>>(tq, tk, tv, tdo, tdq, a, nqs, nos);
    return cudaGetLastError();
  };
#define FA_BWD_CASE(DD, SKK) \
  if (a.D == DD && sk == SKK) return go(bwd_tc_kernel<DD, SKK>);
  FA_BWD_CASE(128, SC_NONE)
  FA_BWD_CASE(128, SC_ALIBI)
  FA_BWD_CASE(128, SC_SOFTCAP)
  FA_BWD_CASE(128, SC_GENERAL)
  FA_BWD_CASE(64, SC_NONE)
  FA_BWD_CASE(64, SC_ALIBI)
  FA_BWD_CASE(64, SC_SOFTCAP)
  FA_BWD_CASE(64, SC_GENERAL)
#undef FA_BWD_CASE
  return cudaErrorInvalidValue;
}

}  // namespace fa
