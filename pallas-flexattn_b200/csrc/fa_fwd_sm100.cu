// FlexAttention forward for B200 (sm_100a): TMA + tcgen05 + TMEM, warp-specialised.
//
// Replaces flash_attention_fwd / flash_attention_fwd_kernel of the reference
// (src/pallas_flexattn/flash_attn.py:59-165).  Same math — online softmax over
// KV tiles, O = softmax(mask(score(QK^T*scale))) V, per-row logsumexp — but:
//   * each CTA owns two 128-row Q tiles of one (b, h) and walks the union of their
//     block-table rows (kv_indices / full_kv_indices); empty tiles are skipped and
//     full tiles do not evaluate the mask (the reference loops over every tile,
//     flash_attn.py:101-104);
//   * S = Q K^T and O += P V run on the 5th-gen tensor cores with the fp32
//     accumulators in TMEM; P is written back to TMEM as bf16 (aliasing S) and fed
//     to the PV MMA straight from TMEM;
//   * the logsumexp is fp32 (the reference stores it in the input dtype,
//     flash_attn.py:144).
//
// Warp roles (384 threads, three warpgroups):
//   warps 0-3  softmax for Q sub-tile 0 (thread = row)     warps 4-7  sub-tile 1
//   warp 8     TMA producer (Q once, then K_j, V_j into an NS-slot ring)
//   warps 9/10 MMA issuers for sub-tiles 0/1 (one thread each); warp 9 owns TMEM; warp 11 idle
// TMEM columns: S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [256+D,256+2D).
// Per kv entry t the issuer of sub-tile i issues PV_i(t) then S_i(t+1), so one
// sub-tile's softmax overlaps the other's tensor-core work.  Because tcgen05 ops of
// one thread complete in issue order, the arrival of S_i(t+1) also proves PV_i(t)
// is done, which is what lets the softmax warps rescale O without another barrier.
// (A single issuing thread for both sub-tiles was measured to leave the tensor pipe
// idle between MMA groups: its serial chain of waits and commits was the bottleneck.)
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "fa_common.cuh"
#include "fa_internal.h"
#include "fa_ptx.cuh"

namespace fa {

namespace {

constexpr int kBM = 128;          // rows of one Q sub-tile
constexpr int kBN = 128;          // rows of one K/V tile
// SPLIT = softmax warps per row quadrant and sub-tile: 1 (thread = row, 128 columns) or 2
// (two warps of the same TMEM lane quadrant share each row, 64 columns each).
//   SPLIT 1: 384 threads = 2 softmax warpgroups + control; the launch gives 168 registers a
//            thread (384 x 168 = 64512), setmaxnreg moves softmax to 216, control to 72.
//   SPLIT 2: 640 threads = 4 softmax warpgroups + control; 96 at launch (640 x 96 = 61440),
//            softmax 104, control 64 (512 x 104 + 128 x 64 = 61440).
// launch_fwd_tc checks the launch allocation against the split before every launch.
template <int SPLIT> struct FwdShape;
template <> struct FwdShape<1> { static constexpr int threads = 384, regs_softmax = 216, regs_ctl = 72; };
template <> struct FwdShape<2> { static constexpr int threads = 640, regs_softmax = 104, regs_ctl = 64; };
// Of every 4 exponential pairs in a full tile, this many run as a polynomial on the FMA
// pipes instead of the MUFU pipe.
#ifndef FA_FWD_EXP_EMU
#define FA_FWD_EXP_EMU 0
#endif
// P is published to the PV MMAs in FA_FWD_P_PARTS parts of 128 / FA_FWD_P_PARTS kv columns.
#ifndef FA_FWD_P_PARTS
#define FA_FWD_P_PARTS 2
#endif
// Softmax ping-pong: -1 chooses per launch, 0 forces it off, 1 forces it on.
#ifndef FA_FWD_PINGPONG
#define FA_FWD_PINGPONG -1
#endif
// P is packed to bf16 with integer ops (1) or with cvt.rn.bf16x2.f32 (0).
#ifndef FA_FWD_INT_PACK
#define FA_FWD_INT_PACK 0
#endif
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows by > 2^8

struct FwdSmemLayout {
  int tile_bytes, q_off, kv_off, bar_off, misc_off, xch_off, cls_off, ent_off, total;
};

// xch: with SPLIT 2, the partner warps' partial row maxima (double-buffered by kv entry
// parity) and, at the end, partial row sums: [2 parity][2 sub-tile][2 half][128] fp32; with kv
// halves, the two sub-tiles' row statistics for the merge ([2 sub-tile][3][128]).
__host__ __device__ inline FwdSmemLayout fwd_smem_layout(int D, int ns, int nkv, bool xch = false) {
  FwdSmemLayout L;
  L.tile_bytes = kBM * D * 2;
  L.q_off = 0;
  L.kv_off = 2 * L.tile_bytes;
  L.bar_off = L.kv_off + ns * L.tile_bytes;
  L.misc_off = L.bar_off + (2 * ns + 10 + 2 * FA_FWD_P_PARTS + 8) * 8;
  L.xch_off = L.misc_off + 16;
  L.cls_off = L.xch_off + (xch ? 2 * 2 * 2 * 128 * 4 : 0);
  L.ent_off = L.cls_off + 4 * nkv;
  L.total = L.ent_off + 4 * nkv + 1024;  // + alignment slack
  return L;
}

template <int D, int SK, int SPLIT>
__global__ void __launch_bounds__(FwdShape<SPLIT>::threads, 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                  const AttnArgs a, const int pingpong, const int tpc) {
  constexpr int CHUNK_BYTES = kBM * 64 * 2;  // one 64-column, 128-byte-swizzled panel
  constexpr int NCHUNK = D / 64;
  constexpr uint32_t TM_S0 = 0, TM_O0 = 256;
  constexpr uint32_t IDESC_S = make_idesc_bf16(kBM, kBN, 0, 0);
  constexpr uint32_t IDESC_PV = make_idesc_bf16(kBM, D, 0, 1);
  constexpr int NT = FwdShape<SPLIT>::threads;
  constexpr int kWarpProd = 8 * SPLIT, kWarpMma0 = kWarpProd + 1;  // issuers kWarpMma0 + i; kWarpMma0 owns TMEM
  static_assert(SPLIT == 1 || FA_FWD_P_PARTS == 2, "with split rows each half publishes one part of P");

  const int NS = a.num_stages;
  const int nkv = a.bt.nkv;
  const FwdSmemLayout L = fwd_smem_layout(D, NS, nkv, SPLIT == 2 || tpc == 4);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L.q_off;
  uint8_t* sKV = smem + L.kv_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* bar_q = bars;
  uint64_t* bar_kv_full = bars + 1;
  uint64_t* bar_kv_empty = bars + 1 + NS;
  uint64_t* bar_s_full = bars + 1 + 2 * NS;   // [2]
  uint64_t* bar_p_full = bar_s_full + 2;       // [2][FA_FWD_P_PARTS]: sub-tile i, part h of P
  uint64_t* bar_o_full = bar_p_full + 2 * FA_FWD_P_PARTS;  // [2]
  uint64_t* bar_teardown = bar_o_full + 2;     // [2]
  uint64_t* bar_turn = bar_teardown + 2;       // [2] softmax ping-pong
  uint64_t* bar_pair = bar_turn + 2;           // [2][4]: the two warps sharing rows (SPLIT 2)
  float* xch = reinterpret_cast<float*>(smem + L.xch_off);
  int* misc = reinterpret_cast<int*>(smem + L.misc_off);
  volatile int* abort_flag = misc;             // misc[0]
  int* n_entries_s = misc + 1;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(misc + 2);
  int* cls = reinterpret_cast<int*>(smem + L.cls_off);
  int* entries = reinterpret_cast<int*>(smem + L.ent_off);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Launch shape `tpc`:
  //   2  sub-tiles 0 and 1 are q tiles 2u and 2u+1 of one head, sharing every K/V load (the
  //      CTA walks the union of their kv lists);
  //   1  q tile u only; sub-tile 1 gets the invalid index nq and idles (twice the CTAs, for
  //      grids that would not fill the SMs);
  //   3  q tile u of heads 2g and 2g+1: both sub-tiles walk the same kv list (tables do not
  //      depend on the head), so neither idles when the list is irregular; each entry loads
  //      K and V of both heads, or once when both heads share a K/V head (grouped queries).
  const bool hpair = tpc == 3;
  const bool kvhalves = tpc == 4;  // one Q tile; sub-tile 0 takes the first half of its kv list, 1 the rest
  const int HU = hpair ? a.H / 2 : a.H;  // head units per batch row
  const int nunits = tpc == 2 ? (a.bt.nq + 1) >> 1 : a.bt.nq;
  int bhu, urank;
  grid_unit_head((int)blockIdx.x, nunits, a.B * HU, &urank, &bhu);
  const int unit = nunits - 1 - urank;  // heaviest (last) q rows first
  const int b = bhu / HU;
  const int h0 = hpair ? 2 * (bhu % HU) : bhu % HU, h1 = hpair ? h0 + 1 : h0;
  const int qt0 = tpc == 2 ? 2 * unit : unit;
  const int qt1 = tpc == 2 ? 2 * unit + 1 : ((hpair || kvhalves) ? unit : a.bt.nq);
  const int hk0 = h0 / (a.H / a.Hkv), hk1 = h1 / (a.H / a.Hkv);
  const bool kv2 = hk1 != hk0;     // two K/V heads: each entry is K0, K1, V0, V1 (else K, V)
  const int LPE = kv2 ? 4 : 2;     // loads per kv entry

  // Block tables: the four list lengths (partial and full, per sub-tile) are independent loads,
  // and each thread fetches its first index of the four lists (taken as one flattened list)
  // before the set-up barrier, so the table reads cost two round trips that overlap the
  // set-up instead of a chain of dependent loads per list.
  int64_t trow0 = 0, trow1 = 0;
  int tcnt[4] = {0, 0, 0, 0};  // partial list of sub-tile 0, of sub-tile 1; full list of 0, of 1
  if (qt0 < a.bt.nq) {
    trow0 = table_head(a.bt, b, h0) * a.bt.nq + qt0;
    tcnt[0] = a.bt.kv_num_blocks ? a.bt.kv_num_blocks[trow0] : 0;
    tcnt[2] = a.bt.full_kv_num_blocks ? a.bt.full_kv_num_blocks[trow0] : 0;
  }
  if (qt1 < a.bt.nq) {
    trow1 = table_head(a.bt, b, h1) * a.bt.nq + qt1;
    tcnt[1] = a.bt.kv_num_blocks ? a.bt.kv_num_blocks[trow1] : 0;
    tcnt[3] = a.bt.full_kv_num_blocks ? a.bt.full_kv_num_blocks[trow1] : 0;
  }
  const int ttot = tcnt[0] + tcnt[1] + tcnt[2] + tcnt[3];
  // kv tile of flattened entry e and its mark: bits 0-1 sub-tile 0, bits 2-3 sub-tile 1;
  // code 1 = partial (mask applied), 2 = full
  auto table_entry = [&](int e, int* mark) -> int {
    int off = e, l = 0;
    if (off >= tcnt[0]) {
      off -= tcnt[0];
      l = 1;
      if (off >= tcnt[1]) {
        off -= tcnt[1];
        l = 2;
        if (off >= tcnt[2]) {
          off -= tcnt[2];
          l = 3;
        }
      }
    }
    *mark = (l >= 2 ? 2 : 1) << (2 * (l & 1));
    return (l >= 2 ? a.bt.full_kv_indices : a.bt.kv_indices)[((l & 1) ? trow1 : trow0) * a.bt.kv_cap + off];
  };
  int my_mark = 0;
  const int my_j = tid < ttot ? table_entry(tid, &my_mark) : -1;

  // ---------------------------------------------------------------- setup
  if (warp == kWarpProd && lane == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar_kv_full + s, 1);
      mbar_init(bar_kv_empty + s, 2);  // released by both MMA issuers
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_s_full + i, 1);
      for (int h = 0; h < FA_FWD_P_PARTS; ++h) mbar_init(bar_p_full + FA_FWD_P_PARTS * i + h, 128);
      mbar_init(bar_o_full + i, 1);
    }
    mbar_init(bar_teardown, 1);
    mbar_init(bar_teardown + 1, 1);
    mbar_init(bar_turn, 128 * SPLIT);
    mbar_init(bar_turn + 1, 128 * SPLIT);
    for (int k = 0; k < 8; ++k) mbar_init(bar_pair + k, 64);
    misc[0] = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    // Q does not depend on the kv lists: its load overlaps the table reads and the set-up.
    const bool has1 = qt1 < a.bt.nq && !kvhalves;  // with kv halves both sub-tiles read Q tile 0
    mbar_arrive_expect_tx(bar_q, (has1 ? 2 : 1) * L.tile_bytes);
    for (int i = 0; i < (has1 ? 2 : 1); ++i)
      for (int c = 0; c < NCHUNK; ++c)
        tma_load_4d(sQ + i * L.tile_bytes + c * CHUNK_BYTES, &tm_q, bar_q, c * 64, (i ? qt1 : qt0) * kBM,
                    i ? h1 : h0, b);
  }
  if (warp == kWarpMma0) {
    tmem_alloc(tmem_base_s, 512);
    tmem_relinquish();
  }
  for (int j = tid; j < nkv; j += NT) cls[j] = 0;
  __syncthreads();

  // Mark the kv tiles each sub-tile visits (a tile listed twice keeps both marks).
  if (my_j >= 0 && my_j < nkv) atomicOr(&cls[my_j], my_mark);
  for (int e = tid + NT; e < ttot; e += NT) {
    int mark;
    const int j = table_entry(e, &mark);
    if (j >= 0 && j < nkv) atomicOr(&cls[j], mark);
  }
  __syncthreads();
  if (warp == kWarpProd) {
    int base = 0;
    for (int j0 = 0; j0 < nkv; j0 += 32) {
      const int j = j0 + lane;
      int c = (j < nkv) ? cls[j] : 0;
      // A tile listed as both partial and full, or one that crosses Tkv, is treated as partial.
      if ((c & 3) == 3) c = (c & ~3) | 1;
      if ((c & 12) == 12) c = (c & ~12) | 4;
      if ((j + 1) * kBN > a.Tkv) {
        if ((c & 3) == 2) c = (c & ~3) | 1;
        if ((c & 12) == 8) c = (c & ~12) | 4;
      }
      const unsigned m = __ballot_sync(0xffffffffu, c != 0);
      if (c) entries[base + __popc(m & ((1u << lane) - 1u))] = j | (c << 24);
      base += __popc(m);
    }
    if (kvhalves) {
      // Both sub-tiles hold the same q tile: the first ceil(n/2) entries go to sub-tile 0, the
      // rest to sub-tile 1, interleaved (e0, e_A, e1, e_A+1, ...) so the producer's in-order
      // loads feed both at once.  The reordered list passes through cls[] (free by now).
      __syncwarp();
      const int A = (base + 1) >> 1, Bn = base - A;
      for (int t = lane; t < base; t += 32) {
        const int src = t < 2 * Bn ? ((t & 1) ? A + (t >> 1) : (t >> 1)) : t - Bn;
        const int e = entries[src];
        const int code = (e >> 24) & 3;  // both sub-tiles carry the same code
        cls[t] = (e & 0xFFFFFF) | ((src < A ? code : code << 2) << 24);
      }
      __syncwarp();
      for (int t = lane; t < base; t += 32) entries[t] = cls[t];
    }
    if (lane == 0) *n_entries_s = base;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_s;
  const int n_ent = *n_entries_s;

  if (warp >= kWarpProd) {
  setmaxnreg_dec<FwdShape<SPLIT>::regs_ctl>();
  if (warp == kWarpProd) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      bool ok = true;
      int issued = 0;  // loads issued so far: per entry K, V (one K/V head) or K0, K1, V0, V1
      for (int t = 0; t < n_ent && ok; ++t) {
        const int j = entries[t] & 0xFFFFFF;
        for (int w = 0; w < LPE && ok; ++w, ++issued) {
          const int slot = issued % NS, use = issued / NS;
          if (!mbar_wait(bar_kv_empty + slot, (use & 1) ^ 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(bar_kv_full + slot, L.tile_bytes);
          const bool is_v = w >= LPE / 2;
          const int kvh = (kv2 && (w & 1)) ? hk1 : hk0;
          for (int c = 0; c < NCHUNK; ++c)
            tma_load_4d(sKV + slot * L.tile_bytes + c * CHUNK_BYTES, is_v ? &tm_v : &tm_k, bar_kv_full + slot,
                        c * 64, j * kBN, kvh, b);
        }
      }
      if (!ok) {
        report_status(a.status, FA_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      // Teardown: make sure no bulk copy into this CTA's shared memory is still in flight.
      volatile int never = 0;
      mbar_wait(bar_q, 0, &never);
      for (int s = 0; s < NS && s < issued; ++s) {
        const int last = s + ((issued - 1 - s) / NS) * NS;  // last load index that used slot s
        mbar_wait(bar_kv_full + s, (last / NS) & 1, &never);
      }
    }
  } else if (warp == kWarpMma0 || warp == kWarpMma0 + 1) {
    // ---------------------------------------------------------------- MMA issuers
    // One issuing thread per Q sub-tile (warp 9: sub-tile 0, warp 10: sub-tile 1), so each
    // thread's serial chain of waits, MMAs and commits covers half the work.  Both walk
    // every kv entry and both commit to the K/V "empty" barriers (initialised with count
    // 2), so a slot is released only after both sub-tiles' MMAs that read it retired.
    // The whole warp runs the loop with warp-uniform values (descriptors stay in uniform
    // registers); elect.sync picks the lane that issues each tcgen05 instruction.
    const int i = warp - kWarpMma0;
    if (n_ent > 0) {
      const uint32_t sQa = smem_u32(sQ), sKVa = smem_u32(sKV);
      int last_t = -1;
      for (int t = 0; t < n_ent; ++t)
        if ((entries[t] >> (24 + 2 * i)) & 3) last_t = t;
      bool ok = mbar_wait_w(bar_q, 0, abort_flag);
      tc_fence_after();
      uint32_t p_phase = 0;
      int pv_count = 0;

      // Descriptors are built once; per K step only the start-address field of the low
      // word moves (see mma_ss_w).  K-major operands (Q, K) use LBO 16 B, the MN-major
      // V operand uses LBO = one 64-column panel; both use SBO = 1024 B (8 swizzled rows).
      const uint64_t dq_base = make_smem_desc(sQa, 16, 1024, SMEM_SWIZZLE_128B);
      const uint32_t desc_hi = (uint32_t)(dq_base >> 32);
      const uint32_t tile16 = (uint32_t)L.tile_bytes >> 4;
      const uint32_t q_lo = (uint32_t)dq_base + (kvhalves ? 0u : i * tile16);  // kv halves share Q tile 0
      const uint32_t k_lo0 = (uint32_t)make_smem_desc(sKVa, 16, 1024, SMEM_SWIZZLE_128B);
      const uint32_t v_lo0 = (uint32_t)make_smem_desc(sKVa, CHUNK_BYTES, 1024, SMEM_SWIZZLE_128B);
      const uint32_t s_dst = tmem_base + TM_S0 + 128 * i, o_dst = tmem_base + TM_O0 + D * i;

      // S_i(t) = Q_i K_t^T (if this sub-tile visits entry t), then release the K slots of entry
      // t.  Every slot is released by both issuers once per use (empty barriers count two
      // arrivals), and a release may only follow the load of the same use, so a slot this
      // sub-tile does not read (the other head's K with two K/V heads, or an entry it skips)
      // is still awaited before it is released: neither thread can release a slot's next use
      // before the other has released the current one.
      auto issue_s = [&](int t, bool part) -> bool {
        for (int w = 0; w < LPE / 2; ++w) {
          const int ld = LPE * t + w, slot = ld % NS;
          if (!mbar_wait_w(bar_kv_full + slot, (ld / NS) & 1, abort_flag)) return false;
          if (part && (!kv2 || w == i)) {
            tc_fence_after();
            const uint32_t klo = k_lo0 + slot * tile16;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              constexpr uint32_t kChunk16 = CHUNK_BYTES >> 4;
              const uint32_t off = (kk >> 2) * kChunk16 + (kk & 3) * 2;
              mma_ss_w(s_dst, q_lo + off, desc_hi, klo + off, desc_hi, IDESC_S, kk > 0);
            }
            tc_commit_w(bar_s_full + i);
          }
          tc_commit_w(bar_kv_empty + slot);
        }
        return true;
      };
      // O_i += P_i V_t (if visited), then release the V slots of entry t (as above).
      auto issue_pv = [&](int t, bool part) -> bool {
        for (int w = 0; w < LPE / 2; ++w) {
          const int ld = LPE * t + LPE / 2 + w, slot = ld % NS;
          if (!mbar_wait_w(bar_kv_full + slot, (ld / NS) & 1, abort_flag)) return false;
          if (part && (!kv2 || w == i)) {
            // P arrives in FA_FWD_P_PARTS parts of kv columns; a part's MMAs start while the
            // softmax warps still compute the next.
            const uint32_t vlo = v_lo0 + slot * tile16;
            const uint32_t acc0 = pv_count > 0 ? 1u : 0u;
            constexpr int KPP = kBN / 16 / FA_FWD_P_PARTS;  // K steps per part
#pragma unroll
            for (int hh = 0; hh < FA_FWD_P_PARTS; ++hh) {
              if (!mbar_wait_w(bar_p_full + FA_FWD_P_PARTS * i + hh, p_phase, abort_flag)) return false;
              tc_fence_after();
#pragma unroll
              for (int kk = KPP * hh; kk < KPP * hh + KPP; ++kk)
                // P of K step kk: kv columns 16kk.. as bf16 pairs; with split rows half h's
                // 64 columns sit at the start of its own S columns (64h)
                mma_ts_w(o_dst, s_dst + (SPLIT == 2 ? (kk >> 2) * 64 + (kk & 3) * 8 : kk * 8),
                         vlo + kk * (2048 >> 4), desc_hi, IDESC_PV, kk > 0 ? 1u : acc0);
            }
            p_phase ^= 1;
            ++pv_count;
            if (t == last_t) tc_commit_w(bar_o_full + i);
          }
          tc_commit_w(bar_kv_empty + slot);
        }
        return true;
      };

      if (ok) ok = issue_s(0, ((entries[0] >> (24 + 2 * i)) & 3) != 0);
      for (int t = 0; t < n_ent && ok; ++t) {
        ok = issue_pv(t, ((entries[t] >> (24 + 2 * i)) & 3) != 0);
        if (ok && t + 1 < n_ent) ok = issue_s(t + 1, ((entries[t + 1] >> (24 + 2 * i)) & 3) != 0);
      }
      if (!ok && lane == 0) {
        report_status(a.status, FA_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      // Teardown: wait (bounded) until every MMA this thread issued has retired.
      tc_commit_w(bar_teardown + i);
      volatile int never = 0;
      mbar_wait(bar_teardown + i, 0, &never);
    }
    __syncwarp();
  }
  } else {
    setmaxnreg_inc<FwdShape<SPLIT>::regs_softmax>();
    // ---------------------------------------------------------------- softmax
    // SPLIT 1: thread = row, all 128 kv columns of a tile.  SPLIT 2: the two warps of a
    // sub-tile that read the same TMEM lane quadrant (w and w + 4 of its 8 warps) share each
    // row: half 0 takes kv columns 0-63, half 1 columns 64-127, and they exchange the partial
    // row maxima per kv entry (and the partial row sums at the end) through shared memory,
    // so two warps per SM sub-partition and sub-tile keep the exponentials flowing.  Each
    // half writes its P into the start of its own S columns and publishes it as one part.
    constexpr int NC = kBN / SPLIT;  // kv columns per thread
    constexpr int DO = D / SPLIT;    // O columns per thread (rescale, epilogue)
    const int i = warp / (4 * SPLIT);
    const int half = SPLIT == 2 ? (warp >> 2) & 1 : 0;
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const int q_row = (i ? qt1 : qt0) * kBM + r;
    const int h = i ? h1 : h0;  // this sub-tile's head
    const uint32_t t_lane = tmem_base + ((uint32_t)(wq * 32) << 16);
    const uint32_t tS = t_lane + TM_S0 + 128 * i + NC * half;  // this thread's S columns (P goes to their start)
    const uint32_t tO = t_lane + TM_O0 + D * i + DO * half;    // this thread's O columns
    uint64_t* pair_bar = bar_pair + 4 * i + wq;
    const ScoreCtx sc = make_score_ctx(a.score, a.scale, h, a.Tkv);
    const MaskCtx mc = make_mask_ctx(a.mask, b, a.Tkv);
    const int qg = q_row + mc.q_off;  // global position of this row (mask and score mods)
    const int dq_val = (mc.flags & FA_MASK_DOCUMENT) && q_row < a.Tq ? __ldg(mc.doc_q + qg) : 0;
    // Causal, window and the Tkv bound intersect to one allowed kv interval [row_lo, row_hi]
    // per row; partial tiles test it with two compares.  Document, tile-table and bitmask
    // predicates (if enabled) are evaluated per element on top.
    int row_lo = mc.kv_off, row_hi = mc.Tkv - 1;  // global kv positions
    if (mc.flags & FA_MASK_CAUSAL) row_hi = min(row_hi, qg);
    if (mc.flags & FA_MASK_WINDOW) {
      if (mc.left >= 0) row_lo = max(row_lo, qg - mc.left);
      if (mc.right >= 0) row_hi = min(row_hi, qg + mc.right);
    }
    // Contiguous documents: the row's document is one kv interval too.
    const bool doc_iv = (mc.flags & FA_MASK_DOCUMENT) && (mc.flags & FA_MASK_DOC_SORTED);
    if (doc_iv) {
      int f, l;
      doc_range(mc.doc_kv, mc.kv_off, mc.Tkv, dq_val, &f, &l);
      row_lo = max(row_lo, f);
      row_hi = min(row_hi, l);
    }
    // A tile table whose cells cover whole 128 x 128 tiles (cell size a multiple of 128, offsets
    // multiples of 128) is tested once per partial tile instead of per element: a tile lies in
    // one cell.
    const bool table_aligned = (mc.flags & FA_MASK_TILE_TABLE) && !(mc.table_block % kBN) && !(mc.q_off % kBN) &&
                               !(mc.kv_off % kBN);
    const bool table_per_elem = (mc.flags & FA_MASK_TILE_TABLE) && !table_aligned;
    const bool per_elem_mask = table_per_elem || (mc.flags & FA_MASK_BITMASK) ||
                               ((mc.flags & FA_MASK_DOCUMENT) && !doc_iv);
    // From here on only row_lo, row_hi, qg, dq_val and per_elem_mask of the mask context stay live.

    // Partner exchange (SPLIT 2): round k writes this thread's value to buffer k & 1, waits
    // for both warps on the pair barrier, reads the partner's.  A buffer is rewritten two
    // rounds later, after the partner has passed the round in between, so it has been read.
    uint32_t xround = 0;
    auto exchange = [&](float v) -> float {
      float* buf = xch + (size_t)(((xround & 1) * 2 + i) * 2) * 128;
      buf[half * 128 + r] = v;
      mbar_arrive(pair_bar);
      const bool got = mbar_wait(pair_bar, xround & 1, abort_flag);
      ++xround;
      return got ? buf[(1 - half) * 128 + r] : v;
    };

    // Turn-taking is compiled only where the host may enable it (no score_mod, or ALiBi).
    constexpr bool PP = SK == SC_NONE || SK == SC_ALIBI;
    float row_max = -INFINITY, row_sum = 0.f;
    uint32_t s_phase = 0;
    int processed = 0;
    bool ok = true;
    for (int t = 0; t < n_ent; ++t) {
      const int e = entries[t];
      const int code = (e >> (24 + 2 * i)) & 3;
      // Ping-pong (when enabled): the two sub-tiles' softmax warps take strict turns (0, 1, 0,
      // 1, ...) for their exponential loops, one turn per kv entry each, visited or not, so one
      // sub-tile's exponentials run while the tensor cores work on the other sub-tile's PV and
      // next S, and the row max (FMA pipe) overlaps the other sub-tile's exponentials (MUFU).
      // Turn k of sub-tile 0 needs sub-tile 1's (k-1)-th hand-over; turn k of sub-tile 1 needs
      // sub-tile 0's k-th.
      const uint32_t turn_parity = i == 0 ? ((t & 1) ^ 1) : (t & 1);
      if (!code) {
        if (PP && pingpong) {
          if (!mbar_wait(bar_turn + i, turn_parity, abort_flag)) { ok = false; break; }
          mbar_arrive(bar_turn + (1 - i));
        }
        continue;
      }
      // global position of this thread's first key in the tile
      const int kvg0 = (e & 0xFFFFFF) * kBN + a.mask.kv_offset + NC * half;
      if (!mbar_wait(bar_s_full + i, s_phase, abort_flag)) { ok = false; break; }
      s_phase ^= 1;
      tc_fence_after();
      float x[NC];
#pragma unroll
      for (int c0 = 0; c0 < NC; c0 += 64) {
        uint32_t r0[32], r1[32];
        tmem_ld32(tS + c0, r0);
        tmem_ld32(tS + c0 + 32, r1);
        tmem_ld_wait();
        reg_pin(r0); reg_pin(r1);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          x[c0 + c] = __uint_as_float(r0[c]);
          x[c0 + 32 + c] = __uint_as_float(r1[c]);
        }
      }
      // Without a score_mod the mask and the max work on the raw dot products, with the softcap
      // on the raw tanh values (both scales are positive), and the scale folds into the
      // exponent's FFMA.
      if constexpr (SK != SC_NONE) {
        const float alibi0 = sc.slope_log2 * (float)(kvg0 - qg);  // ALiBi term of column 0
        const float tanh_k = sc.scale * sc.inv_cap;                 // softcap: tanh argument scale
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          if constexpr (SK == SC_ALIBI) {
            // slope * (kv - q) log2-scaled, as a per-tile base plus the unrolled column
            // index times the slope: two FFMAs, no integer-to-float conversion per element
            x[c] = fmaf(x[c], sc.k_log2, fmaf((float)c, sc.slope_log2, alibi0));
          } else if constexpr (SK == SC_SOFTCAP) {
            // tanh only: cap * log2(e) > 0 scales the max and folds into the exponent's FFMA
            x[c] = fast_tanh(x[c] * tanh_k);
          } else {
            x[c] = score_log2<SK>(x[c], qg, kvg0 + c, sc);
          }
        }
      }
      if (code & 1) {
        const unsigned span = (unsigned)(row_hi - row_lo);
        const int clo = row_lo - kvg0;
        bool kill = row_hi < row_lo;  // the row has no allowed key in any tile
        if (table_aligned)
          kill = kill || !__ldg(a.mask.tile_table + (qg / a.mask.table_block) * a.mask.table_cols +
                                kvg0 / a.mask.table_block);
#pragma unroll
        for (int c = 0; c < NC; ++c)
          if ((unsigned)(c - clo) > span || kill) x[c] = -INFINITY;
        if (per_elem_mask) {
          // Rebuilt from the kernel parameters (constant bank) on the partial tiles that need
          // it, so its pointers and bounds hold no registers across the kv loop.
          const MaskCtx pm = make_mask_ctx(a.mask, b, a.Tkv);
#pragma unroll
          for (int c = 0; c < NC; ++c)
            if (!mask_ok(pm, qg, kvg0 + c, dq_val)) x[c] = -INFINITY;
        }
      }
      // Row max with three-input max: 8 accumulators over columns 0 .. NC-9, then the last 8.
      static_assert(NC == 128 || NC == 64, "the max tree below covers 64 or 128 columns");
      float m8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) m8[k] = fmax3f(x[k], x[8 + k], x[16 + k]);
#pragma unroll
      for (int c = 24; c <= NC - 24; c += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = fmax3f(m8[k], x[c + k], x[c + 8 + k]);
#pragma unroll
      for (int k = 0; k < 8; ++k) m8[k] = fmaxf(m8[k], x[NC - 8 + k]);
      float mloc = fmax3f(fmax3f(m8[0], m8[1], m8[2]), fmax3f(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
      if constexpr (SPLIT == 2) mloc = fmaxf(mloc, exchange(mloc));  // the row's max over all 128 columns
      // Scale folded into the exponent (no score_mod: softmax scale; softcap: cap * log2(e)).
      constexpr bool FOLD = SK == SC_NONE || SK == SC_SOFTCAP;
      const float kfold = SK == SC_NONE ? sc.k_log2 : (SK == SC_SOFTCAP ? sc.cap_log2 : 1.f);
      if constexpr (FOLD) mloc *= kfold;
      if (PP && pingpong && !mbar_wait(bar_turn + i, turn_parity, abort_flag)) { ok = false; break; }
      float alpha = 1.f;
      const bool rescale = mloc > row_max + kRescaleThreshold;
      if (rescale) {
        alpha = ex2_approx(row_max - mloc);  // row_max = -inf gives 0
        row_max = mloc;
      }
      const float m_use = (row_max == -INFINITY) ? 0.f : row_max;
      const float2 kk2 = make_float2(kfold, kfold);
      const float2 nm2 = make_float2(-m_use, -m_use);
      // Rescale O (this thread's DO columns) before any of this entry's P is published (the PV
      // MMAs that read the first part may start before the second is computed); PV(t-1) has
      // retired, since S(t) was committed after it.
      if (processed > 0 && __any_sync(0xffffffffu, rescale)) {
        if constexpr (SPLIT == 1) {
#pragma unroll 1
          for (int c0 = 0; c0 < DO; c0 += 32) {
            uint32_t ov[32];
            tmem_ld32(tO + c0, ov);
            tmem_ld_wait();
            reg_pin(ov);
#pragma unroll
            for (int c = 0; c < 32; ++c) ov[c] = __float_as_uint(__uint_as_float(ov[c]) * alpha);
            tmem_st32(tO + c0, ov);
          }
        } else {  // 16 columns at a time: the logits of the tile are live in registers
#pragma unroll 1
          for (int c0 = 0; c0 < DO; c0 += 16) {
            uint32_t ov[16];
            tmem_ld16(tO + c0, ov);
            tmem_ld_wait();
            reg_pin(ov);
#pragma unroll
            for (int c = 0; c < 16; ++c) ov[c] = __float_as_uint(__uint_as_float(ov[c]) * alpha);
            tmem_st16(tO + c0, ov);
          }
        }
      }
      // Partial sums: four accumulators with whole rows, two with split rows (registers).
      constexpr int NSUM = SPLIT == 2 ? 2 : 4;
      float2 sum2[NSUM];
#pragma unroll
      for (int k = 0; k < NSUM; ++k) sum2[k] = make_float2(0.f, 0.f);
      // Full tiles hold no -inf, so some exponentials may take the polynomial path.
      const bool emu = (code & 1) == 0;
      constexpr int PPT = FA_FWD_P_PARTS / SPLIT;  // parts of P this thread publishes
      constexpr int PW = NC / PPT;                 // kv columns per published part
      constexpr int CW = SPLIT == 2 ? 16 : 32;     // kv columns per TMEM store of P
#pragma unroll
      for (int c0 = 0; c0 < NC; c0 += CW) {
        uint32_t pk[CW / 2];
#pragma unroll
        for (int c = 0; c < CW; c += 2) {
          const float2 y = __ffma2_rn(make_float2(x[c0 + c], x[c0 + c + 1]), kk2, nm2);
          float2 p;
          if (((c >> 1) & 3) < FA_FWD_EXP_EMU && emu) p = exp2_poly2(y);
          else p = make_float2(ex2_approx(y.x), ex2_approx(y.y));
          sum2[(c >> 1) % NSUM] = __fadd2_rn(sum2[(c >> 1) % NSUM], p);
#if FA_FWD_INT_PACK
          pk[c >> 1] = pack_bf16x2_int(p.x, p.y);
#else
          pk[c >> 1] = pack_bf16x2(p.x, p.y);
#endif
        }
        if constexpr (CW == 32) tmem_st16(tS + (c0 >> 1), pk);
        else tmem_st8(tS + (c0 >> 1), pk);
        if ((c0 + CW) % PW == 0) {  // a part of P is written: publish it to the PV MMAs
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(bar_p_full + FA_FWD_P_PARTS * i + half * PPT + c0 / PW);
        }
      }
      if (PP && pingpong) mbar_arrive(bar_turn + (1 - i));  // exponentials issued: the other sub-tile's turn
      float2 s4 = sum2[0];
#pragma unroll
      for (int k = 1; k < NSUM; ++k) s4 = __fadd2_rn(s4, sum2[k]);
      const float sum = s4.x + s4.y;
      row_sum = row_sum * alpha + sum;
      ++processed;
    }
    if (!ok) {
      report_status(a.status, FA_ERR_TIMEOUT);
      *abort_flag = 1;
    }
    // The row's sum over all 128 columns of every tile (both halves scaled by the same maxima).
    if constexpr (SPLIT == 2) {
      if (ok && processed > 0) row_sum += exchange(row_sum);
    }

    // ---------------------------------------------------------------- epilogue
    bool merged = false;
    if constexpr (SPLIT == 1) {
      if (kvhalves) {
        // The two sub-tiles hold the same rows over the two halves of the kv list: exchange the
        // row statistics with the partner warp (same lane quadrant, other sub-tile), then sub-tile
        // i writes output columns [i D/2, (i+1) D/2) of the merged row
        //   o = (O0 2^(m0-m) + O1 2^(m1-m)) / (l0 2^(m0-m) + l1 2^(m1-m)),  m = max(m0, m1),
        // reading both sub-tiles' O columns from TMEM (a sub-tile without entries has no O).
        const bool mine = ok && processed > 0;
        float* st = xch;  // [2 sub-tile][3 field][128]
        st[(i * 3 + 0) * 128 + r] = mine ? row_max : -INFINITY;
        st[(i * 3 + 1) * 128 + r] = mine ? row_sum : 0.f;
        st[(i * 3 + 2) * 128 + r] = mine ? 1.f : 0.f;
        mbar_arrive(bar_pair + wq);
        const bool got = mbar_wait(bar_pair + wq, 0, abort_flag);
        const float m_p = got ? st[((1 - i) * 3 + 0) * 128 + r] : -INFINITY;
        const float l_p = got ? st[((1 - i) * 3 + 1) * 128 + r] : 0.f;
        const bool theirs = got && st[((1 - i) * 3 + 2) * 128 + r] != 0.f;
        if (!got) {
          report_status(a.status, FA_ERR_TIMEOUT);
          *abort_flag = 1;
        }
        const float m_m = mine ? row_max : -INFINITY;
        const float m = fmaxf(m_m, m_p);
        const float a_m = (m_m == -INFINITY) ? 0.f : ex2_approx(m_m - m);
        const float a_p = (m_p == -INFINITY) ? 0.f : ex2_approx(m_p - m);
        const float l = (mine ? row_sum : 0.f) * a_m + l_p * a_p;
        const bool live = l > 0.f;
        const float inv = live ? 1.f / l : 0.f;
        // coefficients and availability of O0 (sub-tile 0) and O1 (sub-tile 1)
        const float c0f = (i == 0 ? a_m : a_p) * inv, c1f = (i == 1 ? a_m : a_p) * inv;
        bool have0 = i == 0 ? mine : theirs, have1 = i == 1 ? mine : theirs;
        if (have0 && !mbar_wait(bar_o_full + 0, 0, abort_flag)) have0 = false;
        if (have1 && !mbar_wait(bar_o_full + 1, 0, abort_flag)) have1 = false;
        // tcgen05.ld is warp-wide: read an O only if every lane may
        have0 = __all_sync(0xffffffffu, have0);
        have1 = __all_sync(0xffffffffu, have1);
        tc_fence_after();
        const int oc0 = i * (D / 2);  // this sub-tile's output columns
        const uint32_t tO0 = t_lane + TM_O0 + oc0, tO1 = t_lane + TM_O0 + D + oc0;
        // The merged rows leave through Q tile 0 (both sub-tiles' S MMAs, its only readers, have
        // retired once both O are complete; without entries the Q load is awaited instead) in the
        // swizzled TMA layout, then by one TMA store per 64-column panel.
        mbar_wait(bar_q, 0, abort_flag);
#pragma unroll 1
        for (int c0 = 0; c0 < D / 2; c0 += 32) {
          uint32_t u0[32] = {}, u1[32] = {};
          if (have0) tmem_ld32(tO0 + c0, u0);
          if (have1) tmem_ld32(tO1 + c0, u1);
          tmem_ld_wait();
          reg_pin(u0);
          reg_pin(u1);
          uint32_t pk[16];
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const float x0 = (have0 ? __uint_as_float(u0[c]) * c0f : 0.f) + (have1 ? __uint_as_float(u1[c]) * c1f : 0.f);
            const float x1 =
                (have0 ? __uint_as_float(u0[c + 1]) * c0f : 0.f) + (have1 ? __uint_as_float(u1[c + 1]) * c1f : 0.f);
            pk[c >> 1] = pack_bf16x2(x0, x1);
          }
          const int col = oc0 + c0;  // first of these 32 output columns
          uint8_t* prow = sQ + (col >> 6) * CHUNK_BYTES + r * 128;
          const int ch0 = (col & 63) >> 3;
#pragma unroll
          for (int v = 0; v < 4; ++v)
            *reinterpret_cast<uint4*>(prow + (((ch0 + v) ^ (r & 7)) << 4)) =
                make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        }
        if (q_row < a.Tq && i == 0)
          a.lse[((int64_t)b * a.H + h) * a.Tq + q_row] = live ? (m + __log2f(l)) * kLn2 : -INFINITY;
        fence_proxy_async_smem();  // the staged rows are visible to the TMA (async proxy)
        named_bar_sync(3, 256);    // both sub-tiles' softmax warps
        if (warp == 0 && lane == 0) {
          for (int c = 0; c < NCHUNK; ++c) tma_store_4d(&tm_o, sQ + c * CHUNK_BYTES, c * 64, qt0 * kBM, h, b);
          bulk_commit_group();
          bulk_wait_read_all();  // shared memory stays valid until the stores have read it
        }
        tc_fence_before();
        merged = true;
      }
    }
    if (!merged) {
    bool have_o = ok && processed > 0;
    if (have_o) {
      have_o = mbar_wait(bar_o_full + i, 0, abort_flag);
      if (!have_o) {
        report_status(a.status, FA_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      tc_fence_after();
    }
    const bool live = row_sum > 0.f;
    const float inv = live ? 1.f / row_sum : 0.f;
    // O leaves through this sub-tile's Q buffer, in the 128-byte-swizzled panel layout of the
    // TMA maps (16-byte chunk c of row r at position c ^ (r & 7)), as one TMA store per 64-column
    // panel.  The buffer is free: O full follows the sub-tile's last S, and a sub-tile without
    // entries still waits for its Q load to land before reusing the buffer.
    const int qt = i ? qt1 : qt0;
    uint8_t* stage = sQ + i * L.tile_bytes;
    if (!have_o) mbar_wait(bar_q, 0, abort_flag);
#pragma unroll 1
    for (int c0 = 0; c0 < DO; c0 += 32) {
      uint32_t ov[32];
      if (have_o) {
        tmem_ld32(tO + c0, ov);
        tmem_ld_wait();
        reg_pin(ov);
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) ov[c] = 0u;
      }
      uint32_t pk[16];
#pragma unroll
      for (int c = 0; c < 32; c += 2)
        pk[c >> 1] = pack_bf16x2(__uint_as_float(ov[c]) * inv, __uint_as_float(ov[c + 1]) * inv);
      const int col = DO * half + c0;  // first of these 32 output columns
      uint8_t* prow = stage + (col >> 6) * CHUNK_BYTES + r * 128;
      const int ch0 = (col & 63) >> 3;
#pragma unroll
      for (int v = 0; v < 4; ++v)
        *reinterpret_cast<uint4*>(prow + (((ch0 + v) ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
    }
    if (q_row < a.Tq && half == 0)
      a.lse[((int64_t)b * a.H + h) * a.Tq + q_row] = live ? (row_max + __log2f(row_sum)) * kLn2 : -INFINITY;
    fence_proxy_async_smem();  // the staged rows are visible to the TMA (async proxy)
    named_bar_sync(1 + i, 128 * SPLIT);
    if (warp == i * 4 * SPLIT && lane == 0 && qt < a.bt.nq) {
      for (int c = 0; c < NCHUNK; ++c) tma_store_4d(&tm_o, stage + c * CHUNK_BYTES, c * 64, qt * kBM, h, b);
      bulk_commit_group();
      bulk_wait_read_all();  // shared memory stays valid until the stores have read it
    }
    tc_fence_before();
    }
  }

  __syncthreads();
  if (warp == kWarpMma0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace

int fwd_tc_max_stages(int D, int nkv) {
  int best = 0;
  for (int ns = 2; ns <= 12; ++ns)
    if (fwd_smem_layout(D, ns, nkv).total <= 227 * 1024) best = ns;
  return best;
}

cudaError_t launch_fwd_tc(const AttnArgs& a_in, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                          const CUtensorMap& to, int tile_cfg, cudaStream_t stream) {
  AttnArgs a = a_in;
  // Rows split over two softmax warps (tile_cfg bits 4-5) only when asked for (the tuner
  // measures both): with the 104-register budget of a split-row thread and the partner
  // exchange, whole rows measured faster on every benchmark config (cfg2 847 vs 733, cfg5
  // 326 vs 295 TFLOP/s).
  const int split = (tile_cfg & 48) == FA_TILE_ROWS_SPLIT ? 2 : 1;
  const int npairs = (a.bt.nq + 1) / 2;
  // Q tiles per CTA (tile_cfg bits 0-1): two unless asked otherwise, or unless pairs would
  // leave most of the SMs idle and single tiles at least double the CTAs.
  int tpc = (tile_cfg & FA_TILE_KV_HALVES) ? 4
            : (tile_cfg & 3) == FA_TILE_Q1 ? 1 : ((tile_cfg & 3) == FA_TILE_HEADS2 ? 3 : 2);
  if (tpc == 3 && a.H % 2) return cudaErrorInvalidValue;  // head pairs need an even head count
  if ((tile_cfg & 3) == 0 && !(tile_cfg & FA_TILE_KV_HALVES)) {
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // Irregular per-tile masks (tile tables, evaluated bitmasks, unsorted document ids) give
    // adjacent q tiles different kv lists: head pairs keep both sub-tiles busy on every entry.
    const bool irregular = (a.mask.flags & (FA_MASK_TILE_TABLE | FA_MASK_BITMASK)) ||
                           ((a.mask.flags & FA_MASK_DOCUMENT) && !(a.mask.flags & FA_MASK_DOC_SORTED));
    // Pairs that would not fill one wave: split each q tile's kv list over the two sub-tiles
    // instead (twice the CTAs, half the longest chain).  Measured on head shards of cfg2 (causal
    // S 4096): 128 pair CTAs 431 -> 545 TFLOP/s; with 256 pair CTAs the pairs stay ahead (800 vs
    // 573), as they do for short rows (cfg3 shards).
    if ((int64_t)npairs * a.B * a.H < (int64_t)sms && a.bt.nq > 1 && split == 1) tpc = 4;
    else if (irregular && a.H % 2 == 0) tpc = 3;
  }
  if (tpc == 4 && split == 2) return cudaErrorInvalidValue;  // kv halves merge whole rows only
  while (a.num_stages > 2 && fwd_smem_layout(a.D, a.num_stages, a.bt.nkv, split == 2 || tpc == 4).total > 227 * 1024)
    --a.num_stages;
  const int smem = fwd_smem_layout(a.D, a.num_stages, a.bt.nkv, split == 2 || tpc == 4).total;
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  const dim3 grid((unsigned)((tpc == 2 ? npairs : a.bt.nq) * a.B * (tpc == 3 ? a.H / 2 : a.H)));
  const int sk = score_kind_of(a.score.flags);
  // Strict softmax turns pay off when the tensor cores bound the loop (head dim 128, no
  // score_mod or only ALiBi's one extra FFMA per score, no per-element mask predicate); a
  // heavier softmax (softcap's tanh) runs better with both warpgroups in flight at once.
  // tile_cfg bits 2-3 override the choice; with one Q tile per CTA there is no second
  // warpgroup to take turns with.
#if FA_FWD_PINGPONG < 0
  const bool per_elem = (a.mask.flags & (FA_MASK_TILE_TABLE | FA_MASK_BITMASK)) ||
                        ((a.mask.flags & FA_MASK_DOCUMENT) && !(a.mask.flags & FA_MASK_DOC_SORTED));
  int pingpong = a.D == 128 && (sk == SC_NONE || sk == SC_ALIBI) && !per_elem;
  if ((tile_cfg & 12) == FA_TILE_SOFTMAX_CONCURRENT) pingpong = 0;
  if ((tile_cfg & 12) == FA_TILE_SOFTMAX_TURNS) pingpong = sk == SC_NONE || sk == SC_ALIBI;  // compiled for these
#else
  int pingpong = FA_FWD_PINGPONG;
#endif
  if (tpc == 1) pingpong = 0;
  auto go = [&](auto kern, auto shape) -> cudaError_t {
    // The register split must fit the launch allocation, or setmaxnreg.inc would wait forever.
    using S = decltype(shape);
    cudaFuncAttributes fa_attr;
    cudaError_t e = cudaFuncGetAttributes(&fa_attr, kern);
    if (e != cudaSuccess) return e;
    const int softmax_threads = S::threads - 128;
    if (fa_attr.numRegs * S::threads < softmax_threads * S::regs_softmax + 128 * S::regs_ctl)
      return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, S::threads, smem, stream>>>(tq, tk, tv, to, a, pingpong, tpc);
    return cudaGetLastError();
  };
#define FA_FWD_CASE(DD, SKK)                                                             \
  if (a.D == DD && sk == SKK)                                                            \
    return split == 2 ? go(fwd_tc_kernel<DD, SKK, 2>, FwdShape<2>{}) : go(fwd_tc_kernel<DD, SKK, 1>, FwdShape<1>{});
  FA_FWD_CASE(128, SC_NONE)
  FA_FWD_CASE(128, SC_ALIBI)
  FA_FWD_CASE(128, SC_SOFTCAP)
  FA_FWD_CASE(128, SC_GENERAL)
  FA_FWD_CASE(64, SC_NONE)
  FA_FWD_CASE(64, SC_ALIBI)
  FA_FWD_CASE(64, SC_SOFTCAP)
  FA_FWD_CASE(64, SC_GENERAL)
#undef FA_FWD_CASE
  return cudaErrorInvalidValue;
}

}  // namespace fa
