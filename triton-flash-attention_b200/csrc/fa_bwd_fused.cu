// fa_bwd_fused.cu -- FlashAttention-2 backward in one pass over the key tiles
// (D <= 64) for B200 (sm_100a).
//
// Produces what the reference's _attn_bwd produces
// (triton_flash_attention/attention.py:383-573): dK and dV as the dK/dV half
// (attention.py:428-505, inner loop :259-308) and dQ as the dQ half
// (attention.py:507-573, inner loop :312-350).  The reference recomputes P
// and dS once for each half; here every (key tile, query tile) pair is
// visited once and yields all three gradients:
//   P^T = exp2(scale*log2(e) * K Q^T - lse2),  dP^T = V dO^T,
//   dS^T = P^T (dP^T - Delta),
//   dV += P^T dO,  dK += dS^T Q  (kept in TMEM for the whole key tile),
//   dQ_part = dS K                (one 128 x D partial per item),
// and the dQ partials are added into an fp32 accumulator [B, Hq, Nq, D] in
// global memory by vector reductions (red.global.add.v4.f32), scaled by the
// softmax scale.  The order of those fp32 additions depends on the
// schedule, so dQ is not bitwise reproducible run to run (dK, dV are: one
// CTA owns a key tile and sums the query heads of its group itself).
//
// Work layout: a persistent CTA per SM walks work tiles of 128 keys of one
// (batch, kv head) in snake order; an item is one (query head of the group,
// 128-row query tile) pair.  Warp roles (512 threads):
//  * warp 0: TMA of K and the Q tiles, plain loads of lse2 / Delta;
//  * warp 3: TMA of V and the dO tiles;
//  * warp 1: one thread issues every tcgen05.mma;
//  * warp 2: owns the TMEM allocation;
//  * warps 4-7 and 8-11: the elementwise warpgroups; warpgroup w takes query
//    half w (64 columns) of every item: P^T = exp2(...) (fp16 / bf16 back
//    into TMEM), then, once dP^T is in, dS^T from the P^T it still holds in
//    registers: packed into TMEM for the dK MMA and written to shared memory
//    (128-byte swizzle) for the dQ MMA, which reads it as an MN-major A
//    operand (dS = (dS^T)^T without a transpose).  Two warps per scheduler
//    share the exponential unit during the exponentials;
//  * warps 12-15: read the dQ partial from TMEM (a warp owns 32 query rows),
//    scale it and turn it through a per-warp shared-memory tile, 32 columns
//    at a time, so that each reduction instruction of the warp covers four
//    whole 128-byte row segments; no barrier beyond the warp and nothing to
//    wait for, the reductions complete on their own.
// TMEM (512 columns): S^T buffers at [0,128) and [128,256) -- P^T of item g
//   packed into columns [0,32) and [64,96) of buffer g & 1 (each query half
//   into the start of its own S^T half, which its warpgroup has read) and the
//   item's dQ partial in columns [64, 64+D) once dV read P^T; dP^T at
//   [256,384) with dS^T packed into [256,288) and [320,352); dV at
//   [384,384+D), dK at [384+D,384+2D).
#include "fa_common.cuh"
#include "fa_kernels.h"
#include "fa_key_tiles.cuh"

namespace fa {

namespace bfz {
constexpr int BM = 128;  // keys per tile
constexpr int BQ = 128;  // query rows per item
constexpr int NUM_THREADS = 512;
#ifndef FA_FUSED_POLY_MASK
#define FA_FUSED_POLY_MASK 0
#endif
#ifndef FA_FUSED_POLY_MASK_D32
#define FA_FUSED_POLY_MASK_D32 2
#endif
constexpr int POLY_MASK = FA_FUSED_POLY_MASK;  // pairs (i & 7) < POLY_MASK use the FMA-pipe exp2 (none: measured fastest)
constexpr int POLY_MASK_D32 = FA_FUSED_POLY_MASK_D32;  // the same at D = 32 (measured)
template <int D>
constexpr int poly_mask() { return D == 32 ? POLY_MASK_D32 : POLY_MASK; }
// Registers per thread: launched at 128 (512 threads); warps 0-3 drop to
// CTRL_REGS and the dQ warpgroup to DQ_REGS, and the two elementwise
// warpgroups rise to SOFT_REGS (ptxas -v shows no spills at this split).
// The shares must add up to at most 512 * 128 = 65536.
constexpr uint32_t LAUNCH_REGS = 128;
constexpr uint32_t CTRL_REGS = 96;
constexpr uint32_t DQ_REGS = 96;
constexpr uint32_t SOFT_REGS = 160;
static_assert(128 * CTRL_REGS + 128 * DQ_REGS + 256 * SOFT_REGS <= NUM_THREADS * LAUNCH_REGS, "register split");

template <int D>
struct Cfg {
  using G = TileGeom<D>;
  static constexpr int NST = 3;
  static constexpr int KV_TILE_BYTES = BM * D * 2;
  static constexpr int Q_TILE_BYTES = BQ * D * 2;
  static constexpr int DS_BYTES = BM * BQ * 2;       // two boxes of 64 query columns, 128-byte swizzle
  static constexpr int DQ_STAGE_BYTES = 4 * 32 * 128;  // per dQ warp: 32 rows x 32 fp32 columns
  static constexpr int OFF_K = 0;                          // 2 buffers
  static constexpr int OFF_V = OFF_K + 2 * KV_TILE_BYTES;  // 2 buffers
  static constexpr int OFF_Q = OFF_V + 2 * KV_TILE_BYTES;
  static constexpr int OFF_DO = OFF_Q + NST * Q_TILE_BYTES;
  static constexpr int OFF_DS = OFF_DO + NST * Q_TILE_BYTES;
  static constexpr int OFF_DQS = OFF_DS + DS_BYTES;
  static constexpr int OFF_LSE = OFF_DQS + DQ_STAGE_BYTES;
  static constexpr int OFF_DELTA = OFF_LSE + NST * BQ * 4;
  static constexpr int OFF_BAR = OFF_DELTA + NST * BQ * 4;
  // kv_full[2], kv_empty[2], full[NST], empty[NST], s_full[2], dp_full, p_ready[2], ds_ready, ds_free,
  // dq_full[2], dq_empty[2], acc_full, acc_empty, mma_done
  static constexpr int NUM_BARS = 2 + 2 + 2 * NST + 2 + 1 + 2 + 1 + 1 + 2 + 2 + 1 + 1 + 1;
  static constexpr int OFF_CTL = OFF_BAR + NUM_BARS * 8;
  static constexpr int OFF_MISC = OFF_CTL + 16;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr int DQ_COL = 64;  // within an S^T buffer
  static constexpr int DP_COL = 256;
  static constexpr int DV_COL = 384;
  static constexpr int DK_COL = 384 + D;
  static_assert(D <= 64, "fused backward is for D <= 64");
  static_assert(DK_COL + D <= TMEM_COLS, "TMEM budget");
  static_assert(OFF_DS % 1024 == 0 && OFF_DQS % 1024 == 0, "swizzled tiles need 1024-byte alignment");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

// Work tiles of BM keys and their BQ-row query items (fa_key_tiles.cuh).
using Tile = KeyTile;
template <bool VL>
__device__ __forceinline__ Tile tile_of(const AttnShape& shp, int t) {
  return key_tile_of<VL, BM, BQ>(shp, t);
}
template <bool VL>
using ItemCursor = KeyItemCursor<VL, BM, BQ>;
}  // namespace bfz

template <int D, int DT, bool VL, bool BITS>
__global__ void __launch_bounds__(bfz::NUM_THREADS, 1)
    fa_bwd_fused_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_do,
                        const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                        float* __restrict__ dq_acc, const AttnShape shp,
                        const float* __restrict__ lse, const float* __restrict__ delta, void* __restrict__ dk_out,
                        const long long dk_sb, const long long dk_sh, const long long dk_sn,
                        void* __restrict__ dv_out, const long long dv_sb, const long long dv_sh,
                        const long long dv_sn, const int accumulate_fp32, const int n_tiles,
                        const MaskBits mk) {
  using namespace bfz;
  using C = Cfg<D>;
  using G = TileGeom<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_saddr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_saddr + 1023u) & ~1023u) - raw_saddr);
  const uint32_t sbase = smem_u32(smem);

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = kv_full + 2;
  uint64_t* full = kv_empty + 2;
  uint64_t* empty = full + C::NST;
  uint64_t* s_full = empty + C::NST;
  uint64_t* dp_full = s_full + 2;
  // Per-buffer barriers (s_full, p_ready, dq_full, dq_empty): phase k of
  // barrier b belongs to item 2k + b, items counted across the CTA's tiles.
  // None can run two phases ahead of its waiters: S^T(g+2) is issued only
  // after the dQ warpgroup read dQ(g), which needs dS^T(g), which needs
  // P^T(g) and dP^T(g) consumed.
  uint64_t* p_ready = dp_full + 1;
  uint64_t* ds_ready = p_ready + 2;
  uint64_t* ds_free = ds_ready + 1;  // one phase per item: the dQ MMA read dS
  uint64_t* dq_full = ds_free + 1;
  uint64_t* dq_empty = dq_full + 2;
  uint64_t* acc_full = dq_empty + 2;  // one phase per non-empty tile: dV, dK complete
  uint64_t* acc_empty = acc_full + 1;  // one phase per non-empty tile: the epilogue read them
  uint64_t* mma_done = acc_empty + 1;
  CtaCtl* ctl_w = reinterpret_cast<CtaCtl*>(smem + C::OFF_CTL);
  volatile CtaCtl* ctl = ctl_w;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  float* s_nlse = reinterpret_cast<float*>(smem + C::OFF_LSE);
  float* s_ndelta = reinterpret_cast<float*>(smem + C::OFF_DELTA);

  const int warp = int(warp_id());
  const int lane = int(lane_id());
  const int group = shp.Hq / shp.Hkv;
  const int cta = int(blockIdx.x);
  const int n_cta = int(gridDim.x);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(kv_full + i, 2);  // K from warp 0, V from warp 3
      mbar_init(kv_empty + i, 1);
      mbar_init(s_full + i, 1);
      mbar_init(p_ready + i, 256);  // both elementwise warpgroups
      mbar_init(dq_full + i, 1);
      mbar_init(dq_empty + i, 128);
    }
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(full + s, 2 + 32);  // two TMA expect_tx arrives + one arrive per lane of warp 0
      mbar_init(empty + s, 1);
    }
    mbar_init(dp_full, 1);
    mbar_init(ds_ready, 256);
    mbar_init(ds_free, 1);
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 256);
    mbar_init(mma_done, 1);
    ctl_w->abort = 0;
    ctl_w->status = shp.status;
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    regs_release<CTRL_REGS>();
    if (warp == 0 || warp == 3) {
      // =================== producer warps ===================
      const bool is_q = warp == 0;
      const CUtensorMap* tmap_kv = is_q ? &tmap_k : &tmap_v;
      const CUtensorMap* tmap_qd = is_q ? &tmap_q : &tmap_do;
      const int kv_off = is_q ? C::OFF_K : C::OFF_V;
      const int qd_off = is_q ? C::OFF_Q : C::OFF_DO;
      if (lane == 0) {
        tma_prefetch_desc(tmap_qd);
        tma_prefetch_desc(tmap_kv);
      }
      // lse2 / Delta of an item's 128 query rows are read with plain loads
      // issued PF items ahead (across tile boundaries): under the TMA stream
      // one L2 round trip would otherwise pace the loop.  Rows past Nq, or
      // rows that see no key, get lse2 = +inf so that their P is 0.
      constexpr int PF = 2;
      float lv[PF + 1][4], dvv[PF + 1][4];
      ItemCursor<VL> ahead{0, 0, {}};
      bool ahead_ok = is_q && ahead.seek(shp, cta, n_cta, n_tiles);
      auto fetch = [&](float (&l)[4], float (&d)[4]) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          l[e] = INFINITY;
          d[e] = 0.f;
        }
        if (!ahead_ok) return;
        const int h = ahead.w.kvh * group + ahead.it / ahead.w.per_head;
        const int q0 = (ahead.w.i_start + ahead.it % ahead.w.per_head) * BQ;
        const long long rowbase = row_stat_index_v<VL>(shp, ahead.w.sq, ahead.w.b, h, 0);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int qi = q0 + e * 32 + lane;
          if (qi < ahead.w.sq.nq) {
            l[e] = lse[rowbase + qi];
            d[e] = delta[rowbase + qi];
          }
        }
        ahead_ok = ahead.next(shp, cta, n_cta, n_tiles);
      };
#pragma unroll
      for (int p = 0; p < PF; ++p) fetch(lv[p], dvv[p]);
      int gi = 0, tcn = 0;  // items and non-empty tiles issued
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int t = snake_unit(cta, k, n_cta, n_tiles);
        if (t >= n_tiles) break;
        const Tile w = tile_of<VL>(shp, t);
        if (w.n_items == 0) continue;
        const int kb = tcn & 1;
        if (tcn >= 2 && !mbar_wait_warp(kv_empty + kb, uint32_t((tcn >> 1) - 1) & 1, ctl, 200)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(kv_full + kb, C::KV_TILE_BYTES);
          for (int bx = 0; bx < G::NBOX; ++bx)
            tma_load_4d(smem + kv_off + kb * C::KV_TILE_BYTES + bx * BM * G::SW, tmap_kv, kv_full + kb,
                        bx * G::BOX, w.sq.k0 + w.kv0, w.kvh, w.sq.tb);
        }
        ++tcn;
        for (int it = 0; it < w.n_items; ++it) {
          if (is_q) fetch(lv[PF], dvv[PF]);
          const int s = gi % C::NST;
          const uint32_t u = uint32_t(gi / C::NST);
          if (u > 0 && !mbar_wait_warp(empty + s, (u - 1) & 1, ctl, 201)) {
            ok = false;
            break;
          }
          const int h = w.kvh * group + it / w.per_head;
          const int q0 = (w.i_start + it % w.per_head) * BQ;
          if (lane == 0) {
            mbar_arrive_expect_tx(full + s, C::Q_TILE_BYTES);
            for (int bx = 0; bx < G::NBOX; ++bx)
              tma_load_4d(smem + qd_off + s * C::Q_TILE_BYTES + bx * BQ * G::SW, tmap_qd, full + s, bx * G::BOX,
                          w.sq.q0 + q0, h, w.sq.tb);
          }
          if (is_q) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float l = lv[0][e] == -INFINITY ? INFINITY : lv[0][e];
              s_nlse[s * BQ + e * 32 + lane] = -l;
              s_ndelta[s * BQ + e * 32 + lane] = -dvv[0][e];
            }
            mbar_arrive(full + s);
#pragma unroll
            for (int p = 0; p < PF; ++p) {
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                lv[p][e] = lv[p + 1][e];
                dvv[p][e] = dvv[p + 1][e];
              }
            }
          }
          ++gi;
        }
      }
      if (lane == 0) {
        for (int j = (tcn > 2 ? tcn - 2 : 0); j < tcn; ++j)
          mbar_wait_drain(kv_full + (j & 1), uint32_t(j >> 1) & 1, ctl, 202);
        for (int j = (gi > C::NST ? gi - C::NST : 0); j < gi; ++j)
          mbar_wait_drain(full + j % C::NST, uint32_t(j / C::NST) & 1, ctl, 203);
      }
    } else if (warp == 1) {
      // =================== tcgen05 MMA issuer ===================
      if (lane == 0) {
        constexpr uint32_t IDESC_ST = idesc_f16_f32(BM, BQ, 0, 0, DT);  // S^T, dP^T: K-major A and B
        constexpr uint32_t IDESC_G = idesc_f16_f32(BM, D, 0, 1, DT);    // dV, dK: A in TMEM, MN-major B
        constexpr uint32_t IDESC_DQ = idesc_f16_f32(BQ, D, 1, 1, DT);   // dQ: MN-major A (dS) and B (K)
        auto q_tile = [&](int g) { return sbase + C::OFF_Q + (g % C::NST) * C::Q_TILE_BYTES; };
        auto do_tile = [&](int g) { return sbase + C::OFF_DO + (g % C::NST) * C::Q_TILE_BYTES; };
        SDesc kd = desc_k_base<D>(sbase + C::OFF_K);
        SDesc vd = desc_k_base<D>(sbase + C::OFF_V);
        SDesc kmn = desc_mn_base<D, BM>(sbase + C::OFF_K);
        // dS as the A operand of dQ: M = 128 queries in two 64-column boxes
        // (LBO apart), K = 128 keys (rows of 128 bytes)
        const SDesc dsd = desc_mn_base<128, BM>(sbase + C::OFF_DS);
        bool ok = true;
        auto issue_s = [&](int g) {  // S^T -> buffer g & 1, once dQ(g - 2) left it
          if (g >= 2 && !mbar_wait(dq_empty + (g & 1), uint32_t((g - 2) >> 1) & 1, ctl, 210)) return false;
          tc_fence_after();
          const SDesc qd = desc_k_base<D>(q_tile(g));
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
            umma_ss(tmem + (g & 1) * 128, sdesc_at(kd, k_major_off<D, BM>(ks)), sdesc_at(qd, k_major_off<D, BQ>(ks)),
                    IDESC_ST, ks > 0);
          umma_commit(s_full + (g & 1));
          return true;
        };
        auto issue_dp = [&](int g) {
          const SDesc dd = desc_k_base<D>(do_tile(g));
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
            umma_ss(tmem + C::DP_COL, sdesc_at(vd, k_major_off<D, BM>(ks)), sdesc_at(dd, k_major_off<D, BQ>(ks)),
                    IDESC_ST, ks > 0);
          umma_commit(dp_full);
        };
        auto wait_full = [&](int g, int site) {
          const bool r = mbar_wait(full + g % C::NST, uint32_t(g / C::NST) & 1, ctl, site);
          tc_fence_after();
          return r;
        };
        // A operand columns of query rows [16ks, 16ks+16): P^T and dS^T are
        // packed in two query halves 64 columns apart
        auto half_col = [](int ks) { return uint32_t((ks >> 2) * 64 + (ks & 3) * 8); };
        int gi = 0, tcn = 0;
        for (int k = 0; ok; ++k) {
          const int t = snake_unit(cta, k, n_cta, n_tiles);
          if (t >= n_tiles) break;
          const int n = tile_of<VL>(shp, t).n_items;
          if (n == 0) continue;
          const int kb = tcn & 1;
          if (!mbar_wait(kv_full + kb, uint32_t(tcn >> 1) & 1, ctl, 211)) { ok = false; break; }
          tc_fence_after();
          kd = desc_k_base<D>(sbase + C::OFF_K + kb * C::KV_TILE_BYTES);
          vd = desc_k_base<D>(sbase + C::OFF_V + kb * C::KV_TILE_BYTES);
          kmn = desc_mn_base<D, BM>(sbase + C::OFF_K + kb * C::KV_TILE_BYTES);
          // the tile's first S^T and dP^T, and the second S^T, run while the
          // warpgroups finish the previous tile
          if (!wait_full(gi, 212) || !issue_s(gi)) { ok = false; break; }
          issue_dp(gi);
          if (n > 1 && (!wait_full(gi + 1, 213) || !issue_s(gi + 1))) { ok = false; break; }
          for (int it = 0; it < n; ++it) {
            const int g = gi + it;
            if (!mbar_wait(p_ready + (g & 1), uint32_t(g >> 1) & 1, ctl, 214)) { ok = false; break; }
            // dV / dK of the previous tile were read by the epilogue
            if (it == 0 && tcn > 0 && !mbar_wait(acc_empty, uint32_t(tcn - 1) & 1, ctl, 215)) { ok = false; break; }
            tc_fence_after();
            {
              const SDesc dd = desc_mn_base<D, BQ>(do_tile(g));
              const uint32_t pa = tmem + (g & 1) * 128;
#pragma unroll
              for (int ks = 0; ks < BQ / 16; ++ks)
                umma_ts(tmem + C::DV_COL, pa + half_col(ks), sdesc_at(dd, mn_major_off<D>(ks)), IDESC_G,
                        (it > 0 || ks > 0) ? 1u : 0u);
            }
            if (!mbar_wait(ds_ready, uint32_t(g) & 1, ctl, 216)) { ok = false; break; }
            tc_fence_after();
            {
              const SDesc qd = desc_mn_base<D, BQ>(q_tile(g));
#pragma unroll
              for (int ks = 0; ks < BQ / 16; ++ks)
                umma_ts(tmem + C::DK_COL, tmem + C::DP_COL + half_col(ks), sdesc_at(qd, mn_major_off<D>(ks)), IDESC_G,
                        (it > 0 || ks > 0) ? 1u : 0u);
            }
            umma_commit(empty + g % C::NST);
            if (it + 1 < n) issue_dp(g + 1);  // its stage was waited for before S^T(g+1)
            {
              const uint32_t dq_t = tmem + (g & 1) * 128 + C::DQ_COL;
#pragma unroll
              for (int ks = 0; ks < BM / 16; ++ks)
                umma_ss(dq_t, sdesc_at(dsd, mn_major_off<128>(ks)), sdesc_at(kmn, mn_major_off<D>(ks)), IDESC_DQ,
                        ks > 0);
              umma_commit(dq_full + (g & 1));
              umma_commit(ds_free);
            }
            if (it + 2 < n && (!wait_full(g + 2, 217) || !issue_s(g + 2))) { ok = false; break; }
          }
          if (!ok) break;
          umma_commit(acc_full);
          umma_commit(kv_empty + kb);
          gi += n;
          ++tcn;
        }
        umma_commit(mma_done);
        mbar_wait_drain(mma_done, 0, ctl, 218);
      }
    }
  } else if (warp < 12) {
    regs_claim<SOFT_REGS>();
    // =================== P^T and dS^T, query half w ===================
    const int w = (warp - 4) / 4;  // query half of every item
    const int wq = warp & 3;
    const int rl = wq * 32 + lane;  // key row within the tile
    const uint32_t lane_base = tmem_addr(tmem, uint32_t(wq * 32), 0);
    const uint64_t c2x2 = f2pack(shp.scale_log2, shp.scale_log2);
    // this thread's row of the swizzled dS^T tile
    const uint32_t ds_row = sbase + C::OFF_DS + uint32_t(rl) * 128u;
    const uint32_t ds_swz = uint32_t(rl & 7);
    int gi = 0, tcn = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int t = snake_unit(cta, k, n_cta, n_tiles);
      if (t >= n_tiles) break;
      const Tile wt = tile_of<VL>(shp, t);
      const long long cmin_base = (long long)wt.kv0 + rl + shp.k_off - shp.q_off;
      // key rows past the batch's keys (the next batch's, when packed) see no query
      const bool key_out = VL && wt.kv0 + rl >= wt.sq.nk;
      // dense boolean mask: this key row's bits of item i's 128 queries (a
      // row past the keys reads the last one), loaded one item ahead
      auto mask_words = [&](int i) -> uint4 {
        const int h = wt.kvh * group + i / wt.per_head;
        const int kr = wt.kv0 + rl < wt.sq.nk ? wt.kv0 + rl : wt.sq.nk - 1;
        const int qi = (wt.i_start + i % wt.per_head) * BQ;
        return __ldg(reinterpret_cast<const uint4*>(mk.bits_t + (long long)wt.b * mk.tsb + (long long)h * mk.tsh +
                                                    (long long)kr * mk.tsn + (qi >> 5)));
      };
      uint4 mw_next;
      if constexpr (BITS) {
        if (wt.n_items > 0) mw_next = mask_words(0);
      }
      for (int it = 0; it < wt.n_items && ok; ++it) {
        const int g = gi + it;
        const int s = g % C::NST;
        const int q0 = (wt.i_start + it % wt.per_head) * BQ;
        // ---- P^T of query half w ----
        uint4 mw;
        if constexpr (BITS) {
          mw = mw_next;
          if (it + 1 < wt.n_items) mw_next = mask_words(it + 1);
        }
        if (!mbar_wait_warp(s_full + (g & 1), uint32_t(g >> 1) & 1, ctl, 220)) { ok = false; break; }
        if (!mbar_wait_warp(full + s, uint32_t(g / C::NST) & 1, ctl, 221)) { ok = false; break; }
        tc_fence_after();
        uint32_t pk_p[32];
        {
          float st[64];
          tmem_ld64(lane_base + uint32_t((g & 1) * 128 + 64 * w), st);
          int cmin = key_out ? 64 : 0;
          if (shp.causal && !key_out) {
            const long long x = cmin_base - q0 - 64 * w;
            cmin = x <= 0 ? 0 : (x > 64 ? 64 : int(x));
          }
          if (cmin > 0) {
#pragma unroll
            for (int c = 0; c < 64; ++c) st[c] = c >= cmin ? st[c] : -INFINITY;
          }
          if (VL && shp.window > 0 && !key_out) {
            // sliding window: queries past this key's window do not see it
            const long long xm = cmin_base + shp.window - 1 - q0 - 64 * w;  // last visible column
            if (xm < 63) {
#pragma unroll
              for (int c = 0; c < 64; ++c) st[c] = c <= xm ? st[c] : -INFINITY;
            }
          }
          if constexpr (BITS) {
            const uint32_t words[2] = {w ? mw.z : mw.x, w ? mw.w : mw.y};
            if ((words[0] & words[1]) != 0xffffffffu) apply_mask_bits<64>(st, words);
          }
          const float4* l4 = reinterpret_cast<const float4*>(s_nlse + s * BQ + 64 * w);
#pragma unroll
          for (int c4 = 0; c4 < 16; ++c4) {
            const float4 nl = l4[c4];
            const int c = c4 * 4;
            const uint64_t x01 = ffma2(f2pack(st[c], st[c + 1]), c2x2, f2pack(nl.x, nl.y));
            const uint64_t x23 = ffma2(f2pack(st[c + 2], st[c + 3]), c2x2, f2pack(nl.z, nl.w));
            const uint64_t e01 = ((2 * c4) & 7) < poly_mask<D>() ? exp2_poly2(x01) : exp2_mufu2(x01);
            const uint64_t e23 = ((2 * c4 + 1) & 7) < poly_mask<D>() ? exp2_poly2(x23) : exp2_mufu2(x23);
            pk_p[c4 * 2] = pack2_f2<DT>(e01);
            pk_p[c4 * 2 + 1] = pack2_f2<DT>(e23);
          }
        }
        // packed into the first 32 columns of this warpgroup's own S^T
        // half, which it has read (the other half may still be unread)
        {
          const uint32_t tP = lane_base + uint32_t((g & 1) * 128 + 64 * w);
          tmem_st16(tP, *reinterpret_cast<uint32_t(*)[16]>(&pk_p[0]));
          tmem_st16(tP + 16, *reinterpret_cast<uint32_t(*)[16]>(&pk_p[16]));
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(p_ready + (g & 1));
        // ---- dS^T of query half w, P from registers ----
        if (!mbar_wait_warp(dp_full, uint32_t(g) & 1, ctl, 223)) { ok = false; break; }
        tc_fence_after();
        uint32_t pk_ds[32];
        {
          const uint32_t tD = lane_base + uint32_t(C::DP_COL + 64 * w);
          float dpt[64];
          tmem_ld64(tD, dpt);
          const float4* d4 = reinterpret_cast<const float4*>(s_ndelta + s * BQ + 64 * w);
#pragma unroll
          for (int c4 = 0; c4 < 16; ++c4) {
            const float4 nd = d4[c4];
            const int c = c4 * 4;
            // dS = P (dP - Delta).  bf16: P widened (two shifts), the product
            // in fp32, one rounding.  fp16: the product in fp16 (widening an
            // fp16 P exactly costs integer work that made the kernel 8%
            // slower for a few percent less error, measured).
            const uint64_t d01f = fadd2(f2pack(dpt[c], dpt[c + 1]), f2pack(nd.x, nd.y));
            const uint64_t d23f = fadd2(f2pack(dpt[c + 2], dpt[c + 3]), f2pack(nd.z, nd.w));
            if constexpr (DT == DT_BF16) {
              pk_ds[c4 * 2] = pack2_f2<DT>(fmul2(widen_bf16x2(pk_p[c4 * 2]), d01f));
              pk_ds[c4 * 2 + 1] = pack2_f2<DT>(fmul2(widen_bf16x2(pk_p[c4 * 2 + 1]), d23f));
            } else {
              pk_ds[c4 * 2] = mul2<DT>(pk_p[c4 * 2], pack2_f2<DT>(d01f));
              pk_ds[c4 * 2 + 1] = mul2<DT>(pk_p[c4 * 2 + 1], pack2_f2<DT>(d23f));
            }
          }
          tmem_st16(tD, *reinterpret_cast<uint32_t(*)[16]>(&pk_ds[0]));
          tmem_st16(tD + 16, *reinterpret_cast<uint32_t(*)[16]>(&pk_ds[16]));
        }
        // the dQ MMA of the previous item has read the dS tile
        if (g > 0 && !mbar_wait_warp(ds_free, uint32_t(g - 1) & 1, ctl, 225)) { ok = false; break; }
        {
          const uint32_t box = ds_row + uint32_t(w) * uint32_t(BM * 128);
#pragma unroll
          for (int c = 0; c < 8; ++c)
            st_shared_v4(box + ((uint32_t(c) ^ ds_swz) << 4), pk_ds[4 * c], pk_ds[4 * c + 1], pk_ds[4 * c + 2],
                         pk_ds[4 * c + 3]);
        }
        tmem_st_wait();
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(ds_ready);
      }
      if (!ok) break;
      // ---- epilogue of the tile: warpgroup 0 stores dV, warpgroup 1 stores dK ----
      if (wt.n_items > 0) {
        if (!mbar_wait_warp(acc_full, uint32_t(tcn) & 1, ctl, 226 + w)) { ok = false; break; }
        tc_fence_after();
      }
      const int kr = wt.kv0 + rl;
      const bool row_ok = kr < wt.sq.nk;
      const float sc = w == 0 ? 1.f : shp.scale;
      const uint32_t tAcc = lane_base + uint32_t(w == 0 ? C::DV_COL : C::DK_COL);
      void* out = w == 0 ? dv_out : dk_out;
      const long long krow = (long long)wt.sq.k0 + kr;
      const long long off0 = w == 0 ? ((long long)wt.sq.tb * dv_sb + (long long)wt.kvh * dv_sh + krow * dv_sn)
                                    : ((long long)wt.sq.tb * dk_sb + (long long)wt.kvh * dk_sh + krow * dk_sn);
#pragma unroll 1
      for (int cc = 0; cc < D / 32; ++cc) {
        float gv[32];
        if (wt.n_items > 0) {
          tmem_ld32(tAcc + cc * 32, gv);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) gv[i] = 0.f;
        }
        if (!row_ok || cc * 32 >= (w == 0 ? shp.v_cols : shp.qk_cols)) continue;
        if (accumulate_fp32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(out) + off0 + cc * 32);
#pragma unroll
          for (int v4 = 0; v4 < 8; ++v4) {
            float4 x = dst[v4];
            x.x += gv[v4 * 4 + 0] * sc;
            x.y += gv[v4 * 4 + 1] * sc;
            x.z += gv[v4 * 4 + 2] * sc;
            x.w += gv[v4 * 4 + 3] * sc;
            dst[v4] = x;
          }
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + off0 + cc * 32);
#pragma unroll
          for (int v8 = 0; v8 < 4; ++v8) {
            uint4 pk;
            pk.x = pack2<DT>(gv[v8 * 8 + 0] * sc, gv[v8 * 8 + 1] * sc);
            pk.y = pack2<DT>(gv[v8 * 8 + 2] * sc, gv[v8 * 8 + 3] * sc);
            pk.z = pack2<DT>(gv[v8 * 8 + 4] * sc, gv[v8 * 8 + 5] * sc);
            pk.w = pack2<DT>(gv[v8 * 8 + 6] * sc, gv[v8 * 8 + 7] * sc);
            dst[v8] = pk;
          }
        }
      }
      if (wt.n_items > 0) {
        tc_fence_before();
        mbar_arrive(acc_empty);
        gi += wt.n_items;
        ++tcn;
      }
    }
  } else {
    regs_release<DQ_REGS>();
    // =================== dQ warpgroup ===================
    const int wq = warp & 3;
    const uint32_t lane_base = tmem_addr(tmem, uint32_t(wq * 32), 0);
    // per warp: a 32-row x 128-byte tile, 16-byte chunk c of row r at
    // chunk c ^ (r & 7) (conflict-free row writes and column-strip reads)
    const uint32_t tile = sbase + C::OFF_DQS + uint32_t(wq) * 4096u;
    const uint32_t my_row = tile + uint32_t(lane) * 128u;
    const uint32_t swz = uint32_t(lane & 7);
    // read side: lane reads chunk lane % 8 of rows 4k + lane / 8
    const int rd_row = lane >> 3, rd_chunk = lane & 7;
    const float sc = shp.scale;
    // rows of one (batch, head) plane of the accumulator
    const long long plane_rows = VL ? shp.total_q : shp.Nq;
    int gi = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int t = snake_unit(cta, k, n_cta, n_tiles);
      if (t >= n_tiles) break;
      const Tile wt = tile_of<VL>(shp, t);
      for (int it = 0; it < wt.n_items; ++it) {
        const int g = gi + it;
        const int h = wt.kvh * group + it / wt.per_head;
        const int q0 = (wt.i_start + it % wt.per_head) * BQ + wq * 32;  // this warp's first query row
        if (!mbar_wait_warp(dq_full + (g & 1), uint32_t(g >> 1) & 1, ctl, 230)) { ok = false; break; }
        tc_fence_after();
        float acc[D];
        const uint32_t tq = lane_base + uint32_t((g & 1) * 128 + C::DQ_COL);
        tmem_ld32(tq, *reinterpret_cast<float(*)[32]>(&acc[0]));
        if constexpr (D == 64) tmem_ld32(tq + 32, *reinterpret_cast<float(*)[32]>(&acc[32]));
        tc_fence_before();
        mbar_arrive(dq_empty + (g & 1));
        // rows past the sequence get nothing (their partials are zero, and
        // in a packed batch they belong to the next sequence)
        float* plane = dq_acc + ((long long)wt.sq.tb * shp.Hq + h) * plane_rows * D;
#pragma unroll
        for (int j = 0; j < D / 32; ++j) {
          __syncwarp();  // the previous strip's reads are done
#pragma unroll
          for (int c = 0; c < 8; ++c)
            st_shared_v4(my_row + ((uint32_t(c) ^ swz) << 4), __float_as_uint(acc[j * 32 + 4 * c] * sc),
                         __float_as_uint(acc[j * 32 + 4 * c + 1] * sc), __float_as_uint(acc[j * 32 + 4 * c + 2] * sc),
                         __float_as_uint(acc[j * 32 + 4 * c + 3] * sc));
          __syncwarp();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const int rr = kk * 4 + rd_row;
            const float4 v = ld_shared_f4(tile + uint32_t(rr) * 128u + ((uint32_t(rd_chunk) ^ uint32_t(rr & 7)) << 4));
            if (q0 + rr < wt.sq.nq)
              red_add_v4(plane + (long long)(wt.sq.q0 + q0 + rr) * D + j * 32 + rd_chunk * 4, v);
          }
        }
      }
      if (!ok) break;
      gi += wt.n_items;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int D, int DT, bool VL, bool BITS = false>
int launch_bwd_fused_t(const BwdArgs& a) {
  using C = bfz::Cfg<D>;
  auto kern = fa_bwd_fused_kernel<D, DT, VL, BITS>;
  // The register split inside the kernel assumes the launch count; a build
  // that allocated a different number must not run (an increase that does
  // not fit would wait forever).
  static int regs_ok = -1;
  if (regs_ok < 0) {
    cudaFuncAttributes fa_attr;
    regs_ok = cudaFuncGetAttributes(&fa_attr, kern) == cudaSuccess && fa_attr.numRegs == int(bfz::LAUNCH_REGS) ? 1 : 0;
  }
  if (!regs_ok) return FA_ERR_LAUNCH;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) != cudaSuccess)
    return FA_ERR_LAUNCH;
  const int n_kt = (a.shape.Nk + bfz::BM - 1) / bfz::BM;
  const int n_tiles = n_kt * a.shape.B * a.shape.Hkv;
  const int sms = device_sm_count();
  const int n_cta = n_tiles < sms ? n_tiles : sms;
  kern<<<dim3(unsigned(n_cta)), bfz::NUM_THREADS, C::SMEM_BYTES, a.stream>>>(
      a.tmap_q, a.tmap_do, a.tmap_k, a.tmap_v, static_cast<float*>(a.dq), a.shape, a.lse, a.delta, a.dk, a.dk_sb,
      a.dk_sh, a.dk_sn,
      a.dv, a.dv_sb, a.dv_sh, a.dv_sn, a.accumulate_fp32, n_tiles, a.mask);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

// Dense and packed (varlen) layouts are separate instantiations, so the
// dense kernels carry no per-batch offset arithmetic.
template <int D, int DT>
int launch_bwd_fused_l(const BwdArgs& a) {
  if (a.mask.bits) return launch_bwd_fused_t<D, DT, false, true>(a);  // dense layout only
  return a.shape.cu_q ? launch_bwd_fused_t<D, DT, true>(a) : launch_bwd_fused_t<D, DT, false>(a);
}

int launch_bwd_fused(const BwdArgs& a, const CUtensorMap& tmap_dq, int D) {
  switch (D) {
    case 32:
      return a.dtype == DT_BF16 ? launch_bwd_fused_l<32, DT_BF16>(a) : launch_bwd_fused_l<32, DT_F16>(a);
    case 64:
      return a.dtype == DT_BF16 ? launch_bwd_fused_l<64, DT_BF16>(a) : launch_bwd_fused_l<64, DT_F16>(a);
    case 128:
      return launch_bwd_fused128(a, tmap_dq);
    default:
      return FA_ERR_UNSUPPORTED_HEAD_DIM;
  }
}

}  // namespace fa
