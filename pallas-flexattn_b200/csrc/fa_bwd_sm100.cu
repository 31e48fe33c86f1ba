// FlexAttention backward for B200 (sm_100a): TMA + tcgen05 + TMEM, warp-specialised.
//
// Replaces the reference's two backward kernels (src/pallas_flexattn/flash_attn.py:
// dK/dV :206-253 and dQ :313-356), which recompute S and P twice (7 tile GEMMs per
// tile pair), with one KV-stationary kernel doing 5 per step:
//   St  = K Q_i^T          dPt = V dO_i^T          (TMEM, fp32)
//   Pt  = exp2(score(St) - lse2_i)   dSt = Pt * (dPt - delta_i) * score'   (registers)
//   dV += Pt dO_i  (A = Pt from TMEM)   dK += dSt Q_i   dQ_i = dS K   (fp32 in TMEM)
// The CTA owns one 128-row kv tile and walks the q tiles of the transposed block table
// (q_indices / full_q_indices) in steps of QR rows, skipping empty tiles; full tiles do
// not evaluate the mask.
//
// A warpgroup drains dQ_i (TMEM -> swizzled shared stage -> TMA reduce-add into an fp32
// accumulator in global memory; fa_bwd scales and converts it afterwards).  TMEM columns:
//   D = 64:   S 128 | dP 128 | dQ 2 x 64 | dV 64 | dK 64   (dQ double-buffered: the drain has
//             a whole step and never holds up the tensor cores)
//   D = 128:  S 128 | dP 128 | dV 128 | dK 128             (full: dQ_i reuses the dP columns
//             once dSt_i is formed, and dPt(t+1) waits for the drain of dQ_t)
// Steps are 128 q rows for both, so every S / dP / dQ product is an N = 128 (or N = D) MMA:
// narrower ones run below the tensor rate, bound by the shared-memory operand reads.
//
// MMA issue order: St(t) dPt(t) dV(t) St(t+1) dQ(t) dK(t) dPt(t+1) dV(t+1) ...  St(t+1)
// goes out as soon as dV(t) has consumed Pt(t) from the S columns, so the next step's
// exponentials can start the moment dSt(t) is written.
//
// Warp roles (512 threads, four warpgroups):
//   WG0, WG1 (warps 0-7)  compute: thread = kv row; WG0 takes q columns [0, QR/2), WG1 the rest
//   WG2 (warps 8-11)      dQ drain: thread = TMEM lane (d for D = 128, q row for D = 64)
//   WG3 (warps 12-15)     warp 12 TMA producer, warp 13 MMA issuer + TMEM owner, 14-15 idle
// Registers: launched at 128 per thread (512 x 128 = 65536); setmaxnreg moves them to
// (D = 128) 152 for WG0/WG1, 128 for WG2 (no change), 80 for WG3, or (D = 64) 176 / 80 / 80.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "fa_common.cuh"
#include "fa_internal.h"
#include "fa_ptx.cuh"

namespace fa {

namespace {

constexpr int kBM = 128;  // kv rows per CTA
constexpr int kBwdThreads = 512;
constexpr int kWarpDq0 = 8, kWarpProd = 12, kWarpMma = 13;
// Register split per warpgroup role (setmaxnreg); each sums to 65536 over 512 threads.
template <int D> struct BwdRegs;
// D = 128: the drain keeps its 128 launch registers to hold three 32-column dQ chunks, so it
// releases the dP columns (and with them the next dPt) one TMA reduce earlier; measured
// 637 -> 660 TFLOP/s on cfg2 against 168 / 96 / 80 with two chunks.
template <> struct BwdRegs<128> { static constexpr int compute = 152, drain = 128, ctl = 80; };
template <> struct BwdRegs<64> { static constexpr int compute = 176, drain = 80, ctl = 80; };
constexpr int kDqStage = 32 * 32 * 4;  // 32 rows x 32 fp32, 128-byte swizzled; one per drain warp

template <int D>
struct BwdCfg {
  static constexpr int QR = 128;                  // q rows per step
  static constexpr int NP = QR / 2;               // q columns per compute thread
  static constexpr bool DQ_OWN = D == 64;         // dQ has TMEM buffers of its own (two)
  static constexpr int PANEL_K = kBM * 128;       // one 64-column swizzle panel of a K/V tile
  static constexpr int PANEL_Q = QR * 128;        // of a Q/dO tile
  static constexpr int PANEL_S = kBM * 128;       // of the dSt tile (rows = kv)
  static constexpr uint32_t TM_S = 0, TM_DP = QR, TM_DQ = DQ_OWN ? 2 * QR : TM_DP,
                            TM_DV = DQ_OWN ? 2 * QR + 2 * D : 2 * QR, TM_DK = TM_DV + D;
  static_assert(TM_DK + D == 512, "TMEM plan must fill the 512 columns");
};

struct BwdSmemLayout {
  int ktile, qtile, k_off, v_off, q_off, o_off, ds_off, dq_off, lse_off, dl_off, bar_off, misc_off, cls_off,
      ent_off, total;
};

__host__ __device__ inline BwdSmemLayout bwd_smem_layout(int D, int nq_st, int no_st, int nq, int G) {
  const int QR = 128;
  BwdSmemLayout L;
  L.ktile = kBM * D * 2;
  L.qtile = QR * D * 2;
  L.k_off = 0;
  L.v_off = L.ktile;
  L.q_off = 2 * L.ktile;
  L.o_off = L.q_off + nq_st * L.qtile;
  L.ds_off = L.o_off + no_st * L.qtile;
  L.dq_off = L.ds_off + kBM * QR * 2;
  L.lse_off = L.dq_off + 4 * kDqStage;
  L.dl_off = L.lse_off + nq_st * QR * 4;
  L.bar_off = L.dl_off + nq_st * QR * 4;
  L.misc_off = L.bar_off + (2 * nq_st + 2 * no_st + 16) * 8;
  L.cls_off = L.misc_off + 16;
  L.ent_off = L.cls_off + 4 * nq;
  L.total = L.ent_off + 4 * nq * G + 1024;  // entries: one 128-row q step per q block and head
  return L;
}

template <int D, int SK>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                  const __grid_constant__ CUtensorMap tm_dq, const __grid_constant__ CUtensorMap tm_dk,
                  const __grid_constant__ CUtensorMap tm_dv, const AttnArgs a, const int NQS, const int NOS) {
  using C = BwdCfg<D>;
  constexpr int QR = C::QR, NP = C::NP;
  constexpr int NCHUNK = D / 64;
  constexpr uint32_t IDESC_SQ = make_idesc_bf16(kBM, QR, 0, 0);  // St, dPt: N = q
  constexpr uint32_t IDESC_KV = make_idesc_bf16(kBM, D, 0, 1);   // dV, dK: A K-major, B MN-major
  constexpr uint32_t IDESC_DQ = make_idesc_bf16(QR, D, 1, 1);   // dQ: A, B MN-major

  const int nq = a.bt.nq;
  const int G = a.H / a.Hkv;  // query heads sharing this CTA's K/V head
  const BwdSmemLayout L = bwd_smem_layout(D, NQS, NOS, nq, G);
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
  uint64_t* bar_dq_full = bar_s_full + 4;   // [2]
  uint64_t* bar_dq_empty = bar_s_full + 6;  // [2]
  uint64_t* bar_dkv_full = bar_s_full + 8;
  uint64_t* bar_teardown = bar_s_full + 9;
  int* misc = reinterpret_cast<int*>(smem + L.misc_off);
  volatile int* abort_flag = misc;
  int* n_entries_s = misc + 1;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(misc + 2);
  int* cls = reinterpret_cast<int*>(smem + L.cls_off);
  int* entries = reinterpret_cast<int*>(smem + L.ent_off);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // One CTA per (kv tile j, b, kv head hk); with grouped-query attention it walks the q
  // tiles of all G query heads of the group, and dK/dV sum over them.
  int j, bhk;  // kv tile (low j first: the most q tiles under causal masks) and (b, K/V head)
  grid_unit_head((int)blockIdx.x, a.bt.nkv, a.B * a.Hkv, &j, &bhk);
  const int b = bhk / a.Hkv, hk = bhk % a.Hkv;
  const int Tq_pad = (a.Tq + 127) / 128 * 128;

  // Block tables of query head g of the group: both list lengths are independent loads, and
  // each thread fetches its first index of the two lists (taken as one) at once, so the reads
  // cost two round trips; head 0's overlap the set-up below.
  struct HeadList {
    int64_t row;
    int np, nf, my_i, my_mark;
  };
  auto head_list = [&](int g) -> HeadList {
    HeadList r;
    r.row = table_head(a.bt, b, hk * G + g) * a.bt.nkv + j;
    r.np = a.bt.q_num_blocks ? a.bt.q_num_blocks[r.row] : 0;
    r.nf = a.bt.full_q_num_blocks ? a.bt.full_q_num_blocks[r.row] : 0;
    r.my_i = -1;
    r.my_mark = 0;
    if (tid < r.np) {
      r.my_i = a.bt.q_indices[r.row * a.bt.q_cap + tid];
      r.my_mark = 1;
    } else if (tid < r.np + r.nf) {
      r.my_i = a.bt.full_q_indices[r.row * a.bt.q_cap + tid - r.np];
      r.my_mark = 2;
    }
    return r;
  };
  HeadList hl = head_list(0);

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
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_dq_full + s, 1);
      mbar_init(bar_dq_empty + s, 128);
    }
    mbar_init(bar_dkv_full, 1);
    mbar_init(bar_teardown, 1);
    misc[0] = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_dq);
    // This CTA's K and V tiles do not depend on the q lists: their load overlaps the table reads.
    mbar_arrive_expect_tx(bar_kv, 2 * L.ktile);
    for (int c = 0; c < NCHUNK; ++c) {
      tma_load_4d(sK + c * C::PANEL_K, &tm_k, bar_kv, c * 64, j * kBM, hk, b);
      tma_load_4d(sV + c * C::PANEL_K, &tm_v, bar_kv, c * 64, j * kBM, hk, b);
    }
  }
  if (warp == kWarpMma) {
    tmem_alloc(tmem_base_s, 512);
    tmem_relinquish();
  }
  int n_built = 0;  // entries built so far (producer warp)
  for (int g = 0; g < G; ++g) {
  if (g > 0) hl = head_list(g);
  for (int i = tid; i < nq; i += kBwdThreads) cls[i] = 0;
  __syncthreads();
  if (hl.my_i >= 0 && hl.my_i < nq) atomicOr(&cls[hl.my_i], hl.my_mark);
  for (int e = tid + kBwdThreads; e < hl.np + hl.nf; e += kBwdThreads) {
    const bool full = e >= hl.np;
    const int i = full ? a.bt.full_q_indices[hl.row * a.bt.q_cap + e - hl.np] : a.bt.q_indices[hl.row * a.bt.q_cap + e];
    if (i >= 0 && i < nq) atomicOr(&cls[i], full ? 2 : 1);
  }
  __syncthreads();
  if (warp == kWarpProd) {
    // Step list: each listed 128-row q block of head g becomes 128 / QR steps of QR rows
    // (steps that start at or past Tq are dropped); entry = step | g << 16 | class << 24
    // (class 1 partial, 2 full).
    constexpr int SPB = 128 / QR;
    int base = n_built;
    for (int i0 = 0; i0 < nq; i0 += 32) {
      const int i = i0 + lane;
      int c = (i < nq) ? cls[i] : 0;
      if (c == 3) c = 1;
      int ns = 0;
      if (c)
        for (int s = 0; s < SPB; ++s) ns += ((i * SPB + s) * QR < a.Tq);
      int incl = ns;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      for (int s = 0; s < ns; ++s) entries[base + incl - ns + s] = (i * SPB + s) | (g << 16) | (c << 24);
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    n_built = base;
    if (lane == 0) *n_entries_s = base;
  }
  __syncthreads();
  }  // heads of the group
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_s;
  const int n_ent = *n_entries_s;

  if (warp >= kWarpProd) {
    setmaxnreg_dec<BwdRegs<D>::ctl>();
    if (warp == kWarpProd) {
      // ---------------------------------------------------------------- TMA producer
      if (lane == 0) {
        const float* lse2 = a.lse2 + (int64_t)b * a.H * Tq_pad;  // rows of head h at + h * Tq_pad
        const float* dl = a.delta + (int64_t)b * a.H * Tq_pad;
        bool ok = true;
        int issued_q = 0, issued_o = 0;
        for (int t = 0; t < n_ent && ok; ++t) {
          const int sub = entries[t] & 0xFFFF, h = hk * G + ((entries[t] >> 16) & 0xFF);
          const int qs = t % NQS, qu = t / NQS;
          if (!mbar_wait(bar_q_empty + qs, (qu & 1) ^ 1, abort_flag)) { ok = false; break; }
          // lse2 and delta ride with Q: the Q slot is released after dK(t), the last reader
          // of Q; the compute warps have read lse2 and delta before dK(t) is issued.
          mbar_arrive_expect_tx(bar_q_full + qs, L.qtile + 2 * QR * 4);
          for (int c = 0; c < NCHUNK; ++c)
            tma_load_4d(sQ + qs * L.qtile + c * C::PANEL_Q, &tm_q, bar_q_full + qs, c * 64, sub * QR, h, b);
          bulk_load(sLse + qs * QR, lse2 + (int64_t)h * Tq_pad + sub * QR, QR * 4, bar_q_full + qs);
          bulk_load(sDl + qs * QR, dl + (int64_t)h * Tq_pad + sub * QR, QR * 4, bar_q_full + qs);
          ++issued_q;
          const int os = t % NOS, ou = t / NOS;
          if (!mbar_wait(bar_o_empty + os, (ou & 1) ^ 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(bar_o_full + os, L.qtile);
          for (int c = 0; c < NCHUNK; ++c)
            tma_load_4d(sO + os * L.qtile + c * C::PANEL_Q, &tm_do, bar_o_full + os, c * 64, sub * QR, h, b);
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
      // The whole warp runs this loop with warp-uniform values (descriptors stay in uniform
      // registers); elect.sync picks the lane that issues each tcgen05 instruction.
      if (n_ent > 0) {
        // Descriptors are built once; per K step only the start-address field of the low
        // word moves (see mma_ss_w).  K-major: LBO 16 B; MN-major: LBO = the operand's
        // 64-column panel stride; SBO = 1024 B for both.  Offsets are in 16-byte units.
        const uint64_t d0 = make_smem_desc(smem_u32(sK), 16, 1024, SMEM_SWIZZLE_128B);
        const uint32_t hi = (uint32_t)(d0 >> 32);
        const uint32_t kmaj = (uint32_t)d0 - ((smem_u32(sK) >> 4) & 0x3FFFu);  // LBO bits only
        const uint32_t mn_k = (uint32_t)make_smem_desc(0, C::PANEL_K, 1024, SMEM_SWIZZLE_128B);
        const uint32_t mn_q = (uint32_t)make_smem_desc(0, C::PANEL_Q, 1024, SMEM_SWIZZLE_128B);
        const uint32_t mn_s = (uint32_t)make_smem_desc(0, C::PANEL_S, 1024, SMEM_SWIZZLE_128B);
        auto lo = [](uint32_t lbo_bits, const void* p) { return lbo_bits + ((smem_u32(p) >> 4) & 0x3FFFu); };
        const uint32_t K_k = lo(kmaj, sK), K_mn = lo(mn_k, sK), V_k = lo(kmaj, sV), S_k = lo(kmaj, sdS),
                       S_mn = lo(mn_s, sdS);
        const uint32_t Q_k0 = lo(kmaj, sQ), Q_mn0 = lo(mn_q, sQ), O_k0 = lo(kmaj, sO), O_mn0 = lo(mn_q, sO);
        const uint32_t qtile16 = (uint32_t)L.qtile >> 4;
        // K-major operand, K step kk of 16 elements along 64-element panels of `panel` bytes
        auto kofs = [](int kk, int panel) { return (uint32_t)((kk >> 2) * (panel >> 4) + (kk & 3) * 2); };
        // MN-major operand, K step kk of 16 rows (two 1024-byte swizzle atoms)
        auto mofs = [](int kk) { return (uint32_t)(kk * (2048 >> 4)); };
        // Pt columns for K step kk (16 q): WG w = kk / (NP/16) holds q [w*NP, (w+1)*NP)
        // packed two per column at TM_S + w*NP.
        auto pcol = [](int kk) { return (uint32_t)((kk / (NP / 16)) * NP + (kk % (NP / 16)) * 8); };

        auto issue_s = [&](int t) -> bool {  // St(t) = K Q^T
          const int qs = t % NQS;
          if (!mbar_wait_w(bar_q_full + qs, (t / NQS) & 1, abort_flag)) return false;
          tc_fence_after();
          const uint32_t Q_k = Q_k0 + qs * qtile16;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_ss_w(tmem_base + C::TM_S, K_k + kofs(kk, C::PANEL_K), hi, Q_k + kofs(kk, C::PANEL_Q), hi, IDESC_SQ,
                      kk > 0);
          tc_commit_w(bar_s_full);
          return true;
        };
        auto issue_dp = [&](int t) -> bool {  // dPt(t) = V dO^T
          const int os = t % NOS;
          if (!mbar_wait_w(bar_o_full + os, (t / NOS) & 1, abort_flag)) return false;
          tc_fence_after();
          const uint32_t O_k = O_k0 + os * qtile16;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_ss_w(tmem_base + C::TM_DP, V_k + kofs(kk, C::PANEL_K), hi, O_k + kofs(kk, C::PANEL_Q), hi,
                      IDESC_SQ, kk > 0);
          tc_commit_w(bar_dp_full);
          return true;
        };

        bool ok = mbar_wait_w(bar_kv, 0, abort_flag);
        tc_fence_after();
        if (ok) ok = issue_s(0);
        if (ok) ok = issue_dp(0);
        for (int t = 0; t < n_ent && ok; ++t) {
          const int qs = t % NQS, os = t % NOS;
          const uint32_t ph = t & 1;
          const uint32_t acc0 = t > 0 ? 1u : 0u;
          // dV += Pt dO
          if (!(ok = mbar_wait_w(bar_p_full, ph, abort_flag))) break;
          tc_fence_after();
          const uint32_t O_mn = O_mn0 + os * qtile16;
#pragma unroll
          for (int kk = 0; kk < QR / 16; ++kk)
            mma_ts_w(tmem_base + C::TM_DV, tmem_base + C::TM_S + pcol(kk), O_mn + mofs(kk), hi, IDESC_KV,
                      kk > 0 ? 1u : acc0);
          tc_commit_w(bar_o_empty + os);  // dPt(t) and dV(t), the readers of dO(t), are issued
          // St(t+1): Pt(t) in the S columns is consumed by dV(t) ahead of it in the pipe
          if (t + 1 < n_ent && !(ok = issue_s(t + 1))) break;
          // dQ(t) = dS K (M = q, N = d), then dK(t).  With buffers of its own, dQ(t) goes to
          // buffer t & 1 once the drain has emptied it; otherwise into the dP columns, which
          // the compute warps have finished reading when they arrive on ds_full.
          if (!(ok = mbar_wait_w(bar_ds_full, ph, abort_flag))) break;
          const int qb = C::DQ_OWN ? (t & 1) : 0;
          if (C::DQ_OWN && t >= 2 && !(ok = mbar_wait_w(bar_dq_empty + qb, ((t >> 1) & 1) ^ 1, abort_flag))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kBM / 16; ++kk)
            mma_ss_w(tmem_base + C::TM_DQ + D * qb, S_mn + mofs(kk), hi, K_mn + mofs(kk), hi, IDESC_DQ, kk > 0);
          tc_commit_w(bar_dq_full + qb);
          const uint32_t Q_mn = Q_mn0 + qs * qtile16;
#pragma unroll
          for (int kk = 0; kk < QR / 16; ++kk)
            mma_ss_w(tmem_base + C::TM_DK, S_k + kofs(kk, C::PANEL_S), hi, Q_mn + mofs(kk), hi, IDESC_KV,
                      kk > 0 ? 1u : acc0);
          tc_commit_w(bar_q_empty + qs);
          // dPt(t+1): the compute warps finished reading dPt(t) before arriving on ds_full;
          // when dQ shares the dP columns, the drain must also have emptied them.
          if (t + 1 < n_ent) {
            if (!C::DQ_OWN && !(ok = mbar_wait_w(bar_dq_empty, t & 1, abort_flag))) break;
            if (!(ok = issue_dp(t + 1))) break;
          }
        }
        if (ok) tc_commit_w(bar_dkv_full);
        if (!ok && lane == 0) {
          report_status(a.status, FA_ERR_TIMEOUT);
          *abort_flag = 1;
        }
        tc_commit_w(bar_teardown);
        volatile int never = 0;
        mbar_wait(bar_teardown, 0, &never);
      }
      __syncwarp();
    }
  } else if (warp >= kWarpDq0) {
    if constexpr (BwdRegs<D>::drain < 128) setmaxnreg_dec<BwdRegs<D>::drain>();  // else keep the launch count
    // ------------------------------------------------------------------ dQ drain (thread = lane)
    // Per step: the D columns of dQ_t for this warp's 32 q rows, in 32-column chunks.  When
    // the drain gates the next dPt (dQ in the dP columns), TMEM loads run AHEAD chunks ahead
    // of the staging (three of the four at D = 128), so the buffer is released after the
    // last load, which needs only the first chunk's staging before it, not the last staging.
    // A chunk is staged 128-byte swizzled in this warp's 4 KB buffer (rewritten only after
    // the previous reduce has read it) and reduce-added by TMA.
    constexpr int AHEAD = C::DQ_OWN ? 1 : (D == 128 ? 3 : 2);  // chunks held in registers
    const int wq = warp & 3;
    uint8_t* stage = sDq + wq * kDqStage;
    bool ok = true;
    for (int t = 0; t < n_ent && ok; ++t) {
      const int sub = entries[t] & 0xFFFF;
      const int bh = b * a.H + hk * G + ((entries[t] >> 16) & 0xFF);  // dQ accumulator row block
      const int qb = C::DQ_OWN ? (t & 1) : 0;
      const uint32_t use = C::DQ_OWN ? (t >> 1) : t;  // completions of this buffer so far
      if (!(ok = mbar_wait(bar_dq_full + qb, use & 1, abort_flag))) break;
      tc_fence_after();
      const uint32_t t_dq = tmem_base + ((uint32_t)(wq * 32) << 16) + C::TM_DQ + D * qb;
      uint32_t v[AHEAD][32];
#pragma unroll
      for (int c = 0; c < AHEAD; ++c) tmem_ld32(t_dq + 32 * c, v[c]);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        reg_pin(v[c % AHEAD]);
        if (c == D / 32 - AHEAD) {  // every chunk is in registers or staged: release the buffer
          tc_fence_before();
          mbar_arrive(bar_dq_empty + qb);
        }
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 8; ++u)
          *reinterpret_cast<uint4*>(stage + lane * 128 + ((u ^ (lane & 7)) << 4)) =
              make_uint4(v[c % AHEAD][4 * u], v[c % AHEAD][4 * u + 1], v[c % AHEAD][4 * u + 2], v[c % AHEAD][4 * u + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_3d(&tm_dq, stage, 32 * c, sub * QR + wq * 32, bh);  // [BH, Tq, D]: x = d, y = q
          bulk_commit_group();
        }
        if (c + AHEAD < D / 32) {  // chunk c is staged: its registers take chunk c + AHEAD
          tmem_ld32(t_dq + 32 * (c + AHEAD), v[c % AHEAD]);
          tmem_ld_wait();
        }
      }
    }
    if (lane == 0) bulk_wait_all();
    if (!ok) {
      report_status(a.status, FA_ERR_TIMEOUT);
      *abort_flag = 1;
    }
  } else {
    setmaxnreg_inc<BwdRegs<D>::compute>();
    // ------------------------------------------------------------------ compute (thread = kv row)
    const int wg = warp >> 2;
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const int kv = j * kBM + r;
    const int cbase = wg * NP;  // first q column (within the step) of this warpgroup
    const uint32_t t_lane = tmem_base + ((uint32_t)(wq * 32) << 16);
    int sc_head = hk * G;  // head the score context below belongs to
    ScoreCtx sc = make_score_ctx(a.score, a.scale, sc_head, a.Tkv);
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
    // Contiguous documents: the kv row's document is one q interval too.
    const bool doc_iv = (mc.flags & FA_MASK_DOCUMENT) && (mc.flags & FA_MASK_DOC_SORTED);
    if (doc_iv && kv < a.Tkv) {
      int f, l;
      doc_range(mc.doc_q, mc.q_off, mc.q_off + a.Tq, __ldg(mc.doc_kv + kvg), &f, &l);
      q_lo = max(q_lo, f);
      q_hi = min(q_hi, l);
    }
    // A tile table whose cells cover whole 128 x 128 tiles (cell size a multiple of 128, offsets
    // multiples of 128) is tested once per partial step instead of per element.
    const bool table_aligned = (mc.flags & FA_MASK_TILE_TABLE) && !(mc.table_block % 128) && !(mc.q_off % 128) &&
                               !(mc.kv_off % 128);
    const bool per_elem_mask = ((mc.flags & FA_MASK_TILE_TABLE) && !table_aligned) || (mc.flags & FA_MASK_BITMASK) ||
                               ((mc.flags & FA_MASK_DOCUMENT) && !doc_iv);
    bool ok = true;
    for (int t = 0; t < n_ent && ok; ++t) {
      const int e = entries[t];
      const int sub = e & 0xFFFF;
      if (G > 1) {  // per-head score parameters (ALiBi slope, bias row)
        const int h = hk * G + ((e >> 16) & 0xFF);
        if (h != sc_head) {
          sc_head = h;
          sc = make_score_ctx(a.score, a.scale, h, a.Tkv);
        }
      }
      const bool partial = ((e >> 24) & 3) == 1;
      const int qs = t % NQS;
      const uint32_t ph = t & 1;
      const float* lse2 = sLse + qs * QR + cbase;
      const float* dl = sDl + qs * QR + cbase;
      const int q0 = sub * QR + cbase;  // local q of this thread's first column

      if (!(ok = mbar_wait(bar_s_full, ph, abort_flag))) break;
      tc_fence_after();
      // p stays fp32 until dSt is formed; each 32-column group of Pt goes back to TMEM (bf16,
      // into already-read S columns) as soon as it is computed.
      float p[NP];
      // Softcap at D = 64 (registers to spare): the derivative 1 - t^2 of each element kept from
      // the P phase as packed fp16 (its 11-bit relative precision on a factor in (0, 1] is
      // finer than the bf16 rounding of dS that follows), instead of recovering t from p with a
      // log2 (a third MUFU operation per element) in the dS phase.
      constexpr bool KEEP_G = SK == SC_SOFTCAP && D == 64;
      uint32_t g2[KEEP_G ? NP / 2 : 1];
#pragma unroll
      for (int hh = 0; hh < NP / 32; ++hh) {
        uint32_t s[32];
        tmem_ld32(t_lane + C::TM_S + cbase + 32 * hh, s);
        // lse2 of the group's 32 q columns: one coalesced load (lane = column), then
        // register shuffles; broadcast loads from shared memory would cost one
        // shared-memory wavefront per 4 values on the pipe the MMAs' operand reads need.
        float l2[32];
        {
          const float lv = lse2[32 * hh + lane];
#pragma unroll
          for (int c = 0; c < 32; ++c) l2[c] = __shfl_sync(0xffffffffu, lv, c);
        }
        tmem_ld_wait();
        reg_pin(s);
        const int qg0 = q0 + 32 * hh + mc.q_off;  // global position of column 0 of this group
        if constexpr (SK == SC_ALIBI) {
          // slope * (kv - q) log2-scaled as a per-group base minus the unrolled column index
          // times the slope: no integer-to-float conversion per element
          const float alibi0 = sc.slope_log2 * (float)(kvg - qg0);
#pragma unroll
          for (int c = 0; c < 32; ++c)
            p[32 * hh + c] = ex2_approx(
                fmaf(__uint_as_float(s[c]), sc.k_log2, fmaf(-(float)c, sc.slope_log2, alibi0)) - l2[c]);
        } else if constexpr (KEEP_G) {
          const float tanh_k = sc.scale * sc.inv_cap;
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const float t0 = fast_tanh(__uint_as_float(s[c]) * tanh_k);
            const float t1 = fast_tanh(__uint_as_float(s[c + 1]) * tanh_k);
            p[32 * hh + c] = ex2_approx(fmaf(sc.cap_log2, t0, -l2[c]));
            p[32 * hh + c + 1] = ex2_approx(fmaf(sc.cap_log2, t1, -l2[c + 1]));
            const __half2 g = __floats2half2_rn(fmaf(-t0, t0, 1.f), fmaf(-t1, t1, 1.f));
            g2[(32 * hh + c) >> 1] = *reinterpret_cast<const uint32_t*>(&g);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c)
            p[32 * hh + c] = ex2_approx(score_log2<SK>(__uint_as_float(s[c]), qg0 + c, kvg, sc) - l2[c]);
        }
        if (partial) {
          const unsigned span = (unsigned)(q_hi - q_lo);
          const int clo = q_lo - qg0;
          bool kill = q_hi < q_lo;
          if (table_aligned)
            kill = kill || !__ldg(mc.table + (qg0 / mc.table_block) * mc.table_cols + kvg / mc.table_block);
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if ((unsigned)(c - clo) > span || kill) p[32 * hh + c] = 0.f;
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
        tmem_st16(t_lane + C::TM_S + cbase + 16 * hh, pk);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar_p_full);

      // dPt(t) is issued after dK(t-1), so when it completes dQ(t-1) and dK(t-1) have read
      // dSt(t-1) and the dSt buffer may be rewritten.
      if (!(ok = mbar_wait(bar_dp_full, ph, abort_flag))) break;
      tc_fence_after();
#pragma unroll
      for (int hh = 0; hh < NP / 32; ++hh) {
        uint32_t dp[32];
        tmem_ld32(t_lane + C::TM_DP + cbase + 32 * hh, dp);
        float dl32[32];  // delta of the group's columns, distributed as lse2 above
        {
          const float dv = dl[32 * hh + lane];
#pragma unroll
          for (int c = 0; c < 32; ++c) dl32[c] = __shfl_sync(0xffffffffu, dv, c);
        }
        tmem_ld_wait();
        reg_pin(dp);
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const int cc = 32 * hh + c;
          float d0 = p[cc] * (__uint_as_float(dp[c]) - dl32[c]);
          float d1 = p[cc + 1] * (__uint_as_float(dp[c + 1]) - dl32[c + 1]);
          if constexpr (KEEP_G) {
            const float2 g = __half22float2(*reinterpret_cast<const __half2*>(&g2[cc >> 1]));
            d0 *= g.x;
            d1 *= g.y;
          } else if constexpr (SK == SC_SOFTCAP || SK == SC_GENERAL) {
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
        const int qq = cbase + 32 * hh;  // first q column (within the step) of this group
        uint8_t* ds_row = sdS + (qq >> 6) * C::PANEL_S + r * 128;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int unit = ((qq & 63) >> 3) + u;  // 16-byte unit within the 128-byte row
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
    if constexpr (D == 128) {
      // dV and dK leave through the V and K buffers (every MMA that reads them has retired when
      // dK/dV full completes; a CTA without entries waits for its K/V load to land instead), in
      // the 128-byte-swizzled panel layout of the TMA maps (16-byte chunk c of row r at position
      // c ^ (r & 7)), as one TMA store per 64-column panel; rows past Tkv are not written.
      if (!have) mbar_wait(bar_kv, 0, abort_flag);
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        const float mul = which ? a.scale : 1.f;
        uint8_t* stage = which ? sK : sV;
        const uint32_t tcol = which ? C::TM_DK : C::TM_DV;
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
          uint32_t pk[16];
#pragma unroll
          for (int c = 0; c < 32; c += 2)
            pk[c >> 1] = pack_bf16x2(__uint_as_float(v[c]) * mul, __uint_as_float(v[c + 1]) * mul);
          uint8_t* prow = stage + (c0 >> 6) * C::PANEL_K + r * 128;
          const int ch0 = (c0 & 63) >> 3;
#pragma unroll
          for (int u = 0; u < 4; ++u)
            *reinterpret_cast<uint4*>(prow + (((ch0 + u) ^ (r & 7)) << 4)) =
                make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
      }
      fence_proxy_async_smem();  // the staged rows are visible to the TMA (async proxy)
      named_bar_sync(1, 256);    // both compute warpgroups
      if (tid == 0) {
        for (int c = 0; c < NCHUNK; ++c) {
          tma_store_4d(&tm_dv, sV + c * C::PANEL_K, c * 64, j * kBM, hk, b);
          tma_store_4d(&tm_dk, sK + c * C::PANEL_K, c * 64, j * kBM, hk, b);
        }
        bulk_commit_group();
        bulk_wait_read_all();  // shared memory stays valid until the stores have read it
      }
    } else {
      // Head dim 64: the rows go straight to global memory (the CTAs are short, and waiting for
      // the stores to read shared memory before exit measured slower: cfg5 backward -4 %).
      __nv_bfloat16* dvr = reinterpret_cast<__nv_bfloat16*>(a.dv.ptr) + (int64_t)b * a.dv.stride_b +
                           (int64_t)hk * a.dv.stride_h + (int64_t)kv * a.dv.stride_t;
      __nv_bfloat16* dkr = reinterpret_cast<__nv_bfloat16*>(a.dk.ptr) + (int64_t)b * a.dk.stride_b +
                           (int64_t)hk * a.dk.stride_h + (int64_t)kv * a.dk.stride_t;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        const float mul = which ? a.scale : 1.f;
        __nv_bfloat16* dst = which ? dkr : dvr;
        const uint32_t tcol = which ? C::TM_DK : C::TM_DV;
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
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

bool pick_stages(int D, int nq, int G, int* nqs, int* nos) {
  const int cand[7][2] = {{4, 4}, {4, 3}, {3, 3}, {3, 2}, {2, 2}, {2, 1}, {0, 0}};
  for (int c = 0; cand[c][0]; ++c)
    if (bwd_smem_layout(D, cand[c][0], cand[c][1], nq, G).total <= 227 * 1024) {
      *nqs = cand[c][0];
      *nos = cand[c][1];
      return true;
    }
  return false;
}

}  // namespace

int bwd_tc_max_stages(int D, int nq, int G) {
  int a = 0, b = 0;
  return pick_stages(D, nq, G, &a, &b) ? a : 0;
}

int bwd_tc_q_rows(int D) { return D == 128 ? BwdCfg<128>::QR : BwdCfg<64>::QR; }

cudaError_t launch_bwd_tc(const AttnArgs& a, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                          const CUtensorMap& tdo, const CUtensorMap& tdq, const CUtensorMap& tdk,
                          const CUtensorMap& tdv, cudaStream_t stream) {
  int nqs = 0, nos = 0;
  const int G = a.H / a.Hkv;
  if (!pick_stages(a.D, a.bt.nq, G, &nqs, &nos)) return cudaErrorInvalidValue;
  if (a.num_stages >= 2 && a.num_stages < nqs) nqs = a.num_stages;
  if (nos > nqs) nos = nqs;
  const int smem = bwd_smem_layout(a.D, nqs, nos, a.bt.nq, G).total;
  const dim3 grid((unsigned)(a.bt.nkv * a.B * a.Hkv));
  const int sk = score_kind_of(a.score.flags);
  auto go = [&](auto kern, auto regs) -> cudaError_t {
    // The register split must fit the launch allocation, or setmaxnreg.inc would wait forever.
    using R = decltype(regs);
    cudaFuncAttributes fa_attr;
    cudaError_t e = cudaFuncGetAttributes(&fa_attr, kern);
    if (e != cudaSuccess) return e;
    if (fa_attr.numRegs * kBwdThreads < 2 * 128 * R::compute + 128 * R::drain + 128 * R::ctl)
      return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, kBwdThreads, smem, stream>>>(tq, tk, tv, tdo, tdq, tdk, tdv, a, nqs, nos);
    return cudaGetLastError();
  };
#define FA_BWD_CASE(DD, SKK) \
  if (a.D == DD && sk == SKK) return go(bwd_tc_kernel<DD, SKK>, BwdRegs<DD>{});
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
