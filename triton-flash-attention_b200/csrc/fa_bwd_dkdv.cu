// fa_bwd_dkdv.cu -- FlashAttention-2 backward, dK/dV half, for B200 (sm_100a).
//
// Computes what the dK/dV half of the reference's _attn_bwd produces
// (triton_flash_attention/attention.py:428-505, inner loop :258-308):
//   P^T = exp2(scale*log2(e) * K Q^T - lse2),  dP^T = V dO^T,
//   dS^T = P^T (dP^T - Delta),  dV = sum P^T dO,  dK = scale * sum dS^T Q,
// where the sums run over every query row that sees the key and, for GQA,
// over every query head of the key's group.  The reference sums the group
// with fp16 atomics (attention.py:503-505); here one CTA owns a key tile and
// loops over the group's heads itself, so the sum is deterministic.
// Layout of the work (D = 128 kernel; the D <= 64 kernel below differs in
// the item width):
//  * a persistent CTA per SM walks work tiles of 128 keys of one (batch, kv
//    head) in snake order; K and V of a tile stay resident in shared memory
//    for the tile's whole sweep and are double-buffered across tiles;
//  * warps 0 and 3 stream (query head, 64-row query tile) items: Q and dO
//    tiles by TMA, and the items' lse2 / Delta values with plain loads by the
//    32 lanes of warp 0;
//  * warp 1 (one thread) issues tcgen05.mma: S^T = K Q^T and dP^T = V dO^T
//    into one of two TMEM buffers, then dV += P^T dO and dK += dS^T Q with
//    P^T, dS^T read from TMEM (fp16) and Q, dO read as MN-major operands;
//  * warps 4-7 and 8-11 take alternate items (two TMEM buffers), one thread
//    per key row, and write P^T and dS^T back to TMEM;
//  * after a tile's last item warpgroup 0 stores dV and warpgroup 1 stores
//    dK while the MMA issuer already runs the next tile's first S^T / dP^T.
// TMEM: buffer w: S^T at [128w, 128w+64), dP^T at [128w+64, 128w+128);
//       dV at [256, 256+D), dK at [256+D, 256+2D).
#include "fa_common.cuh"
#include "fa_kernels.h"
#include "fa_key_tiles.cuh"

namespace fa {

namespace bkv {

constexpr int BM = dkdv_cfg::BM;  // keys per tile (MMA M)
constexpr int BQ = dkdv_cfg::BQ;  // query rows per item (MMA N, then K)
constexpr int NUM_THREADS = 384;
// Registers per thread: launched at 168 (384 threads); warps 0-3 (producers,
// MMA issuer, TMEM owner) drop to CTRL_REGS and the two P^T / dS^T
// warpgroups rise to SOFT_REGS.  128 * CTRL_REGS + 256 * SOFT_REGS must not
// exceed 384 * 168 = 64512.
constexpr uint32_t LAUNCH_REGS = 168;
constexpr uint32_t CTRL_REGS = 64;
constexpr uint32_t SOFT_REGS = 216;
static_assert(128 * CTRL_REGS + 256 * SOFT_REGS <= NUM_THREADS * LAUNCH_REGS, "register split");

template <int D>
struct Cfg {
  using G = TileGeom<D>;
  static constexpr int NST = 3;  // Q / dO stages (two K / V buffers take 4 x 32 KB at D = 128)
  static constexpr int KV_TILE_BYTES = BM * D * 2;
  static constexpr int Q_TILE_BYTES = BQ * D * 2;
  static constexpr int OFF_K = 0;                                  // 2 buffers
  static constexpr int OFF_V = OFF_K + 2 * KV_TILE_BYTES;          // 2 buffers
  static constexpr int OFF_Q = OFF_V + 2 * KV_TILE_BYTES;          // NST stages
  static constexpr int OFF_DO = OFF_Q + NST * Q_TILE_BYTES;        // NST stages
  static constexpr int OFF_LSE = OFF_DO + NST * Q_TILE_BYTES;      // NST x BQ floats
  static constexpr int OFF_DELTA = OFF_LSE + NST * BQ * 4;         // NST x BQ floats
  static constexpr int OFF_BAR = OFF_DELTA + NST * BQ * 4;
  // kv_full[2], kv_empty[2], full[NST], empty[NST], st_full[2], ds_ready[2], acc_full, acc_empty, mma_done
  static constexpr int NUM_BARS = 2 + 2 + 2 * NST + 2 + 2 + 1 + 1 + 1;
  static constexpr int OFF_CTL = OFF_BAR + NUM_BARS * 8;
  static constexpr int OFF_MISC = OFF_CTL + 16;
  static constexpr int SMEM_USED = OFF_MISC + 16 + 1024;
  static constexpr int SMEM_BYTES = SMEM_USED;
  static constexpr int TMEM_COLS = 512;
  static constexpr int DV_COL = 256;
  static constexpr int DK_COL = 256 + D;
  static_assert(DK_COL + D <= TMEM_COLS, "TMEM budget");
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
}  // namespace bkv

template <int D, int DT, bool VL, bool BITS, bool DROP>
__global__ void __launch_bounds__(bkv::NUM_THREADS, 1)
    fa_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_do,
                       const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                       const AttnShape shp, const float* __restrict__ lse, const float* __restrict__ delta,
                       void* __restrict__ dk_out, const long long dk_sb, const long long dk_sh, const long long dk_sn,
                       void* __restrict__ dv_out, const long long dv_sb, const long long dv_sh, const long long dv_sn,
                       const int accumulate_fp32, const int n_tiles, const MaskBits mk,
                       const DropArgs dr) {
  using namespace bkv;
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
  // per item parity w (items alternate between the warpgroups, counted
  // across the CTA's tiles)
  uint64_t* st_full = empty + C::NST;
  uint64_t* ds_ready = st_full + 2;
  uint64_t* acc_full = ds_ready + 2;   // one phase per non-empty tile: dV, dK complete
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
    }
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(full + s, 2 + 32);  // two TMA expect_tx arrives + one arrive per lane of warp 0
      mbar_init(empty + s, 1);
    }
    for (int w = 0; w < 2; ++w) {
      mbar_init(st_full + w, 1);
      mbar_init(ds_ready + w, 128);
    }
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
      // Warp 0 loads K and the Q tiles and writes lse2 / Delta; warp 3 loads V
      // and the dO tiles.  One thread's TMA loads are processed one after
      // another, so the two streams come from two threads.
      const bool is_q = warp == 0;
      const CUtensorMap* tmap_kv = is_q ? &tmap_k : &tmap_v;
      const CUtensorMap* tmap_qd = is_q ? &tmap_q : &tmap_do;
      const int kv_off = is_q ? C::OFF_K : C::OFF_V;
      const int qd_off = is_q ? C::OFF_Q : C::OFF_DO;
      if (lane == 0) {
        tma_prefetch_desc(tmap_qd);
        tma_prefetch_desc(tmap_kv);
      }
      // lse2 / Delta of an item's 64 query rows are read with plain loads
      // issued PF items ahead (across tile boundaries): under the TMA stream one
      // L2 round trip would otherwise pace the loop.  Rows past Nq, or rows
      // that see no key, get lse2 = +inf so that their P is 0.
      constexpr int PF = 2;
      float lv[PF + 1][2], dvv[PF + 1][2];
      ItemCursor<VL> ahead{0, 0, {}};
      bool ahead_ok = is_q && ahead.seek(shp, cta, n_cta, n_tiles);
      auto fetch = [&](float (&l)[2], float (&d)[2]) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          l[e] = INFINITY;
          d[e] = 0.f;
        }
        if (!ahead_ok) return;
        const int h = ahead.w.kvh * group + ahead.it / ahead.w.per_head;
        const int q0 = (ahead.w.i_start + ahead.it % ahead.w.per_head) * BQ;
        const long long rowbase = row_stat_index_v<VL>(shp, ahead.w.sq, ahead.w.b, h, 0);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int qi = q0 + lane * 2 + e;
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
        if (tcn >= 2 && !mbar_wait_warp(kv_empty + kb, uint32_t((tcn >> 1) - 1) & 1, ctl, 60)) { ok = false; break; }
        if (lane == 0) {
          mbar_arrive_expect_tx(kv_full + kb, C::KV_TILE_BYTES);
          for (int bx = 0; bx < G::NBOX; ++bx)
            tma_load_4d(smem + kv_off + kb * C::KV_TILE_BYTES + bx * BM * G::SW, tmap_kv, kv_full + kb, bx * G::BOX,
                        w.sq.k0 + w.kv0, w.kvh, w.sq.tb);
        }
        ++tcn;
        for (int it = 0; it < w.n_items; ++it) {
          if (is_q) fetch(lv[PF], dvv[PF]);
          const int s = gi % C::NST;
          const uint32_t u = uint32_t(gi / C::NST);
          if (u > 0 && !mbar_wait_warp(empty + s, (u - 1) & 1, ctl, 61)) { ok = false; break; }
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
            for (int e = 0; e < 2; ++e) {
              const float l = lv[0][e] == -INFINITY ? INFINITY : lv[0][e];
              s_nlse[s * BQ + lane * 2 + e] = -l;
              s_ndelta[s * BQ + lane * 2 + e] = -dvv[0][e];
            }
            mbar_arrive(full + s);
#pragma unroll
            for (int p = 0; p < PF; ++p) {
#pragma unroll
              for (int e = 0; e < 2; ++e) {
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
          mbar_wait_drain(kv_full + (j & 1), uint32_t(j >> 1) & 1, ctl, 62);
        for (int j = (gi > C::NST ? gi - C::NST : 0); j < gi; ++j)
          mbar_wait_drain(full + j % C::NST, uint32_t(j / C::NST) & 1, ctl, 63);
      }
    } else if (warp == 1) {
      // =================== tcgen05 MMA issuer ===================
      if (lane == 0) {
        constexpr uint32_t IDESC_ST = idesc_f16_f32(BM, BQ, 0, 0, DT);
        constexpr uint32_t IDESC_G = idesc_f16_f32(BM, D, 0, 1, DT);
        SDesc kd = desc_k_base<D>(sbase + C::OFF_K);
        SDesc vd = desc_k_base<D>(sbase + C::OFF_V);
        auto issue_st = [&](int g) {  // S^T, dP^T of item g -> buffer g & 1
          const int w = g & 1;
          const int s = g % C::NST;
          const SDesc qd = desc_k_base<D>(sbase + C::OFF_Q + s * C::Q_TILE_BYTES);
          const SDesc dd = desc_k_base<D>(sbase + C::OFF_DO + s * C::Q_TILE_BYTES);
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
            umma_ss(tmem + w * 128, sdesc_at(kd, k_major_off<D, BM>(ks)), sdesc_at(qd, k_major_off<D, BQ>(ks)), IDESC_ST,
                    ks > 0);
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
            umma_ss(tmem + w * 128 + 64, sdesc_at(vd, k_major_off<D, BM>(ks)), sdesc_at(dd, k_major_off<D, BQ>(ks)),
                    IDESC_ST, ks > 0);
          umma_commit(st_full + w);
        };
        auto issue_grad = [&](int g, bool acc) {
          const int w = g & 1;
          const int s = g % C::NST;
          const SDesc qd = desc_mn_base<D, BQ>(sbase + C::OFF_Q + s * C::Q_TILE_BYTES);
          const SDesc dd = desc_mn_base<D, BQ>(sbase + C::OFF_DO + s * C::Q_TILE_BYTES);
          const uint32_t acc0 = acc ? 1u : 0u;
          umma_ts(tmem + C::DV_COL, tmem + w * 128, sdesc_at(dd, 0), IDESC_G, acc0);
#pragma unroll
          for (int ks = 1; ks < BQ / 16; ++ks)
            umma_ts(tmem + C::DV_COL, tmem + w * 128 + ks * 8, sdesc_at(dd, mn_major_off<D>(ks)), IDESC_G, 1u);
          umma_ts(tmem + C::DK_COL, tmem + w * 128 + 64, sdesc_at(qd, 0), IDESC_G, acc0);
#pragma unroll
          for (int ks = 1; ks < BQ / 16; ++ks)
            umma_ts(tmem + C::DK_COL, tmem + w * 128 + 64 + ks * 8, sdesc_at(qd, mn_major_off<D>(ks)), IDESC_G, 1u);
        };
        auto wait_full = [&](int g, int site) {
          const bool r = mbar_wait(full + g % C::NST, uint32_t(g / C::NST) & 1, ctl, site);
          tc_fence_after();
          return r;
        };
        int gi = 0, tcn = 0;
        bool ok = true;
        for (int k = 0; ok; ++k) {
          const int t = snake_unit(cta, k, n_cta, n_tiles);
          if (t >= n_tiles) break;
          const int n = tile_of<VL>(shp, t).n_items;
          if (n == 0) continue;
          const int kb = tcn & 1;
          if (!mbar_wait(kv_full + kb, uint32_t(tcn >> 1) & 1, ctl, 70)) { ok = false; break; }
          tc_fence_after();
          kd = desc_k_base<D>(sbase + C::OFF_K + kb * C::KV_TILE_BYTES);
          vd = desc_k_base<D>(sbase + C::OFF_V + kb * C::KV_TILE_BYTES);
          // the tile's first two items run while the warpgroups finish the
          // previous tile
          if (!wait_full(gi, 71)) { ok = false; break; }
          issue_st(gi);
          if (n > 1) {
            if (!wait_full(gi + 1, 72)) { ok = false; break; }
            issue_st(gi + 1);
          }
          for (int it = 0; it < n; ++it) {
            const int g = gi + it;
            if (!mbar_wait(ds_ready + (g & 1), uint32_t(g >> 1) & 1, ctl, 73)) { ok = false; break; }
            // dV / dK of the previous tile were read by the epilogue
            if (it == 0 && tcn > 0 && !mbar_wait(acc_empty, uint32_t(tcn - 1) & 1, ctl, 76)) { ok = false; break; }
            tc_fence_after();
            issue_grad(g, it > 0);
            umma_commit(empty + g % C::NST);
            if (it + 2 < n) {
              if (!wait_full(g + 2, 74)) { ok = false; break; }
              issue_st(g + 2);
            }
          }
          if (!ok) break;
          umma_commit(acc_full);
          umma_commit(kv_empty + kb);
          gi += n;
          ++tcn;
        }
        umma_commit(mma_done);
        mbar_wait_drain(mma_done, 0, ctl, 75);
      }
    }
  } else {
    regs_claim<SOFT_REGS>();
    // =================== P^T / dS^T warpgroups ===================
    const int w = (warp - 4) / 4;  // item parity and TMEM buffer of this warpgroup
    const int wq = warp & 3;
    const int rl = wq * 32 + lane;  // key row within the tile
    const uint32_t tS = tmem_addr(tmem, uint32_t(wq * 32), uint32_t(w * 128));
    const float c2 = shp.scale_log2;
    const uint64_t c2x2 = f2pack(c2, c2);
    int gi = 0, tcn = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int t = snake_unit(cta, k, n_cta, n_tiles);
      if (t >= n_tiles) break;
      const Tile wt = tile_of<VL>(shp, t);
      // causal: key row rl sees query column c of an item at rows q0.. iff
      // c >= cmin_base - q0
      const long long cmin_base = (long long)wt.kv0 + rl + shp.k_off - shp.q_off;
      // key rows past the batch's keys (the next batch's, when packed) see no query
      const bool key_out = VL && wt.kv0 + rl >= wt.sq.nk;
      // dense boolean mask: this key row's bits of item i's queries (a row
      // past the keys reads the last one), loaded one item of this
      // warpgroup ahead
      auto mask_words = [&](int i) -> uint2 {
        const int h = wt.kvh * group + i / wt.per_head;
        const int kr = wt.kv0 + rl < wt.sq.nk ? wt.kv0 + rl : wt.sq.nk - 1;
        const int qi = (wt.i_start + i % wt.per_head) * BQ;
        return __ldg(reinterpret_cast<const uint2*>(mk.bits_t + (long long)wt.b * mk.tsb + (long long)h * mk.tsh +
                                                    (long long)kr * mk.tsn + (qi >> 5)));
      };
      const int it0 = (gi & 1) == w ? 0 : 1;
      uint2 mw_next;
      if constexpr (BITS) {
        if (it0 < wt.n_items) mw_next = mask_words(it0);
      }
      // this warpgroup's items of the tile: global parity w
      for (int it = it0; it < wt.n_items; it += 2) {
        const int g = gi + it;
        const int s = g % C::NST;
        uint2 mw;
        if constexpr (BITS) {
          mw = mw_next;
          if (it + 2 < wt.n_items) mw_next = mask_words(it + 2);
        }
        if (!mbar_wait_warp(st_full + w, uint32_t(g >> 1) & 1, ctl, 80 + w)) { ok = false; break; }
        // the stage's lse2/Delta values: their phase completed before st_full
        if (!mbar_wait_warp(full + s, uint32_t(g / C::NST) & 1, ctl, 82 + w)) { ok = false; break; }
        tc_fence_after();
        float st[BQ], dpt[BQ];
        tmem_ld64(tS, st);
        tmem_ld64(tS + 64, dpt);
        const int q0 = (wt.i_start + it % wt.per_head) * BQ;
        // dropout: P~ = Z P feeds dV, dS = P (Z r dP - Delta); this key row
        // uses bytes (k & 1) and 2 + (k & 1) of each 2 x 2 block word
        uint32_t drop_k2 = 0;
        if constexpr (DROP)
          drop_k2 = drop_key2(drop_key_bh(dr, wt.b * shp.Hq + wt.kvh * group + it / wt.per_head), q0, wt.kv0 + rl);
        int cmin = key_out ? BQ : 0;
        if (shp.causal && !key_out) {
          const long long x = cmin_base - q0;
          cmin = x <= 0 ? 0 : (x > BQ ? BQ : int(x));
        }
        if (cmin > 0) {  // causal diagonal: queries before this key are invisible
#pragma unroll
          for (int c = 0; c < BQ; ++c) st[c] = c >= cmin ? st[c] : -INFINITY;
        }
        if (VL && shp.window > 0 && !key_out) {
          // sliding window: queries past this key's window do not see it
          const long long xm = cmin_base + shp.window - 1 - q0;  // last visible column
          if (xm < BQ - 1) {
#pragma unroll
            for (int c = 0; c < BQ; ++c) st[c] = c <= xm ? st[c] : -INFINITY;
          }
        }
        if constexpr (BITS) {
          const uint32_t words[2] = {mw.x, mw.y};
          if ((words[0] & words[1]) != 0xffffffffu) apply_mask_bits<BQ>(st, words);
        }
        // stage values are stored negated: -lse2 and -Delta
        const float4* l4 = reinterpret_cast<const float4*>(s_nlse + s * BQ);
        const float4* d4 = reinterpret_cast<const float4*>(s_ndelta + s * BQ);
        uint32_t pk_p[BQ / 2], pk_ds[BQ / 2];
#pragma unroll
        for (int c4 = 0; c4 < BQ / 4; ++c4) {
          const float4 nl = l4[c4];
          const float4 nd = d4[c4];
          const int c = c4 * 4;
          const uint64_t e01 = exp2_mufu2(ffma2(f2pack(st[c], st[c + 1]), c2x2, f2pack(nl.x, nl.y)));
          const uint64_t e23 = exp2_mufu2(ffma2(f2pack(st[c + 2], st[c + 3]), c2x2, f2pack(nl.z, nl.w)));
          const uint32_t p01 = pack2_f2<DT>(e01);
          const uint32_t p23 = pack2_f2<DT>(e23);
          if constexpr (DROP) {
            // the words of query pairs (c, c+1) and (c+2, c+3) for this key row pair
            const int kb = rl & 1;  // kv0 is even
            uint32_t w01, w23;
            shared_words(drop_word(drop_k2, q0 + c + 2 * kb, wt.kv0 + rl), kb, w01, w23);
            const uint32_t sel = kb ? keep_sel(1, 3) : keep_sel(0, 2);
            const uint32_t tt = (256u - dr.t) * 0x10001u;
            const uint32_t m01 = keep_mask2(w01, sel, tt);
            const uint32_t m23 = keep_mask2(w23, sel, tt);
            const uint64_t r2 = f2pack(dr.r, dr.r);
            const uint32_t n01 = pack2_f2<DT>(f2pack(nd.x, nd.y)), n23 = pack2_f2<DT>(f2pack(nd.z, nd.w));
            const uint32_t k01 = pack2_f2<DT>(ffma2(f2pack(dpt[c], dpt[c + 1]), r2, f2pack(nd.x, nd.y)));
            const uint32_t k23 = pack2_f2<DT>(ffma2(f2pack(dpt[c + 2], dpt[c + 3]), r2, f2pack(nd.z, nd.w)));
            pk_p[c4 * 2] = p01 & m01;
            pk_p[c4 * 2 + 1] = p23 & m23;
            pk_ds[c4 * 2] = mul2<DT>(p01, (k01 & m01) | (n01 & ~m01));
            pk_ds[c4 * 2 + 1] = mul2<DT>(p23, (k23 & m23) | (n23 & ~m23));
          } else {
            // dS = P (dP - Delta) in fp32, rounded once (attention.py:300-305)
            pk_p[c4 * 2] = p01;
            pk_p[c4 * 2 + 1] = p23;
            pk_ds[c4 * 2] = pack2_f2<DT>(fmul2(e01, fadd2(f2pack(dpt[c], dpt[c + 1]), f2pack(nd.x, nd.y))));
            pk_ds[c4 * 2 + 1] = pack2_f2<DT>(fmul2(e23, fadd2(f2pack(dpt[c + 2], dpt[c + 3]), f2pack(nd.z, nd.w))));
          }
        }
        tmem_st16(tS, *reinterpret_cast<uint32_t(*)[16]>(&pk_p[0]));
        tmem_st16(tS + 16, *reinterpret_cast<uint32_t(*)[16]>(&pk_p[16]));
        tmem_st16(tS + 64, *reinterpret_cast<uint32_t(*)[16]>(&pk_ds[0]));
        tmem_st16(tS + 80, *reinterpret_cast<uint32_t(*)[16]>(&pk_ds[16]));
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(ds_ready + w);
      }
      if (!ok) break;
      // ---- epilogue of the tile: warpgroup 0 stores dV, warpgroup 1 stores dK ----
      if (wt.n_items > 0) {
        if (!mbar_wait_warp(acc_full, uint32_t(tcn) & 1, ctl, 84 + w)) { ok = false; break; }
        tc_fence_after();
      }
      const int kr = wt.kv0 + rl;
      const bool row_ok = kr < wt.sq.nk;
      const float sc = w == 0 ? (DROP ? dr.r : 1.f) : shp.scale;  // dV of dropped-out P~ carries r
      const uint32_t tAcc = tmem_addr(tmem, uint32_t(wq * 32), uint32_t(w == 0 ? C::DV_COL : C::DK_COL));
      void* out = w == 0 ? dv_out : dk_out;
      const long long krow = (long long)wt.sq.k0 + kr;
      const long long off0 = w == 0 ? ((long long)wt.sq.tb * dv_sb + (long long)wt.kvh * dv_sh + krow * dv_sn)
                                    : ((long long)wt.sq.tb * dk_sb + (long long)wt.kvh * dk_sh + krow * dk_sn);
#pragma unroll 1
      for (int cc = 0; cc < D / 32; ++cc) {
        float gv[32];
        if (wt.n_items > 0) {
          tmem_ld32(tAcc + cc * 32, gv);
          if (cc == D / 32 - 1) {
            // both accumulators are read: the next tile may overwrite them
            tc_fence_before();
            mbar_arrive(acc_empty);
          }
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
        gi += wt.n_items;
        ++tcn;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// D <= 64: persistent kernel with 128-query items.  At D <= 64 an N = 64 MMA
// runs at ~70% of the tensor rate (measured: M128 x N x K16 takes
// max(N/2, ~45) cycles), so the items here are 128 query rows wide (S^T, dP^T
// are N = 128 MMAs at full rate).
// One CTA per SM walks its share of the work tiles (128 keys of one batch and
// kv head each) back to back: K/V are double-buffered, so the next tile's K/V
// load, its first S^T / dP^T MMAs and its first exponentials overlap the
// current tile's last items and its dK/dV epilogue.  Measured before this
// change, one CTA per tile spent ~7k of its ~60k cycles on the start-up and
// the epilogue that nothing overlapped.
// The two elementwise warpgroups are specialised by phase: warpgroup 0 turns
// S^T into P^T (the exponentials) for whole items, warpgroup 1 turns dP^T and
// P^T into dS^T, one item behind.  S^T is double-buffered in TMEM; the MMA
// thread issues dV(i) as soon as P^T(i) is published and dK(i), dP^T(i+1),
// S^T(i+2) once dS^T(i) is.
// TMEM: S^T buffers at [0,128) and [128,256), dP^T at [256,384),
//       dV at [384, 384+D), dK at [384+D, 384+2D).
// P^T of query columns [64h, 64h+64) is packed into its S^T buffer's columns
// [64h, 64h+32), dS^T likewise into dP^T's columns [256+64h, 256+64h+32):
// each half is written after it was read.
namespace bkvw {
constexpr int BM = 128;   // keys per tile
constexpr int BQ = 128;   // query rows per item
constexpr int NUM_THREADS = 384;
constexpr int POLY_MASK = 3;  // pairs (i & 7) < 3 use the FMA-pipe exp2 (measured fastest here)

template <int D>
struct Cfg {
  using G = TileGeom<D>;
  static constexpr int NST = 4;
  static constexpr int KV_TILE_BYTES = BM * D * 2;
  static constexpr int Q_TILE_BYTES = BQ * D * 2;
  static constexpr int OFF_K = 0;                          // 2 buffers
  static constexpr int OFF_V = OFF_K + 2 * KV_TILE_BYTES;  // 2 buffers
  static constexpr int OFF_Q = OFF_V + 2 * KV_TILE_BYTES;
  static constexpr int OFF_DO = OFF_Q + NST * Q_TILE_BYTES;
  static constexpr int OFF_LSE = OFF_DO + NST * Q_TILE_BYTES;
  static constexpr int OFF_DELTA = OFF_LSE + NST * BQ * 4;
  static constexpr int OFF_BAR = OFF_DELTA + NST * BQ * 4;
  // kv_full[2], kv_empty[2], full[NST], empty[NST], s_full[2], dp_full, p_ready[2], ds_ready,
  // acc_full, acc_empty, mma_done
  static constexpr int NUM_BARS = 2 + 2 + 2 * NST + 2 + 1 + 2 + 1 + 1 + 1 + 1;
  static constexpr int OFF_CTL = OFF_BAR + NUM_BARS * 8;
  static constexpr int OFF_MISC = OFF_CTL + 16;
  static constexpr int SMEM_USED = OFF_MISC + 16 + 1024;
  static constexpr int SMEM_BYTES = SMEM_USED;
  static constexpr int TMEM_COLS = 512;
  static constexpr int DP_COL = 256;
  static constexpr int DV_COL = 384;
  static constexpr int DK_COL = 384 + D;
  static_assert(D <= 64, "wide dK/dV path is for D <= 64");
  static_assert(DK_COL + D <= TMEM_COLS, "TMEM budget");
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
}  // namespace bkvw

template <int D, int DT, bool VL, bool BITS>
__global__ void __launch_bounds__(bkvw::NUM_THREADS, 1)
    fa_bwd_dkdv_wide_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_do,
                            const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                            const AttnShape shp, const float* __restrict__ lse, const float* __restrict__ delta,
                            void* __restrict__ dk_out, const long long dk_sb, const long long dk_sh,
                            const long long dk_sn, void* __restrict__ dv_out, const long long dv_sb,
                            const long long dv_sh, const long long dv_sn, const int accumulate_fp32,
                            const int n_tiles, const MaskBits mk) {
  using namespace bkvw;
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
  // p_ready is per S^T buffer: phase k of p_ready[b] belongs to item 2k+b, so
  // it cannot run two phases ahead of its waiters (item i+2's S^T is issued
  // only after dS^T(i) -- and so P^T(i) -- was consumed).  Items are counted
  // across the CTA's tiles.
  uint64_t* p_ready = dp_full + 1;
  uint64_t* ds_ready = p_ready + 2;
  uint64_t* acc_full = ds_ready + 1;   // one phase per non-empty tile: dV, dK complete
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
    }
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(full + s, 2 + 32);  // two TMA expect_tx arrives + one arrive per lane of warp 0
      mbar_init(empty + s, 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_full + 1, 1);
    mbar_init(dp_full, 1);
    mbar_init(p_ready, 128);
    mbar_init(p_ready + 1, 128);
    mbar_init(ds_ready, 128);
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

  if (warp == 0 || warp == 3) {
    // =================== producer warps ===================
    // Warp 0 loads K and the Q tiles and writes lse2 / Delta; warp 3 loads V
    // and the dO tiles.  One thread's TMA loads are processed one after
    // another, so the two streams come from two threads.
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
    // issued two items ahead (across tiles): under the TMA stream one L2
    // round trip (~1-2k cycles) would otherwise pace the loop.  Rows past Nq,
    // or rows that see no key, get lse2 = +inf so that their P is 0.
    constexpr int PF = 2;
    float lv[PF + 1][4], dv[PF + 1][4];
    int pf_k = 0, pf_it = 0;  // prefetch cursor: tile round k, item it
    Tile pf_w = tile_of<VL>(shp, snake_unit(cta, 0, n_cta, n_tiles) < n_tiles ? snake_unit(cta, 0, n_cta, n_tiles) : 0);
    bool pf_live = snake_unit(cta, 0, n_cta, n_tiles) < n_tiles;
    auto pf_skip_empty = [&]() {
      while (pf_live && pf_it >= pf_w.n_items) {
        pf_it = 0;
        ++pf_k;
        const int t = snake_unit(cta, pf_k, n_cta, n_tiles);
        pf_live = t < n_tiles;
        if (pf_live) pf_w = tile_of<VL>(shp, t);
      }
    };
    auto fetch = [&](float (&l)[4], float (&d)[4]) {
      pf_skip_empty();
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        l[e] = INFINITY;
        d[e] = 0.f;
      }
      if (!pf_live || !is_q) return;
      const int h = pf_w.kvh * group + pf_it / pf_w.per_head;
      const int q0 = (pf_w.i_start + pf_it % pf_w.per_head) * BQ;
      const long long rowbase = row_stat_index_v<VL>(shp, pf_w.sq, pf_w.b, h, 0);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = q0 + e * 32 + lane;
        if (qi < pf_w.sq.nq) {
          l[e] = lse[rowbase + qi];
          d[e] = delta[rowbase + qi];
        }
      }
      ++pf_it;
    };
#pragma unroll
    for (int p = 0; p < PF; ++p) fetch(lv[p], dv[p]);
    int gi = 0, tcn = 0;  // items and non-empty tiles issued
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int t = snake_unit(cta, k, n_cta, n_tiles);
      if (t >= n_tiles) break;
      const Tile w = tile_of<VL>(shp, t);
      if (w.n_items == 0) continue;
      const int kb = tcn & 1;
      if (tcn >= 2 && !mbar_wait_warp(kv_empty + kb, uint32_t((tcn >> 1) - 1) & 1, ctl, 160)) { ok = false; break; }
      if (lane == 0) {
        mbar_arrive_expect_tx(kv_full + kb, C::KV_TILE_BYTES);
        for (int bx = 0; bx < G::NBOX; ++bx)
          tma_load_4d(smem + kv_off + kb * C::KV_TILE_BYTES + bx * BM * G::SW, tmap_kv, kv_full + kb, bx * G::BOX,
                      w.sq.k0 + w.kv0, w.kvh, w.sq.tb);
      }
      ++tcn;
      for (int it = 0; it < w.n_items; ++it) {
        fetch(lv[PF], dv[PF]);
        const int s = gi % C::NST;
        const uint32_t u = uint32_t(gi / C::NST);
        if (u > 0 && !mbar_wait_warp(empty + s, (u - 1) & 1, ctl, 161)) { ok = false; break; }
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
            s_ndelta[s * BQ + e * 32 + lane] = -dv[0][e];
          }
          mbar_arrive(full + s);
        }
#pragma unroll
        for (int p = 0; p < PF; ++p) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            lv[p][e] = lv[p + 1][e];
            dv[p][e] = dv[p + 1][e];
          }
        }
        ++gi;
      }
    }
    if (lane == 0) {
      for (int j = (tcn > 2 ? tcn - 2 : 0); j < tcn; ++j)
        mbar_wait_drain(kv_full + (j & 1), uint32_t(j >> 1) & 1, ctl, 162);
      for (int j = (gi > C::NST ? gi - C::NST : 0); j < gi; ++j)
        mbar_wait_drain(full + j % C::NST, uint32_t(j / C::NST) & 1, ctl, 163);
    }
  } else if (warp == 1) {
    // =================== tcgen05 MMA issuer ===================
    if (lane == 0) {
      constexpr uint32_t IDESC_ST = idesc_f16_f32(BM, BQ, 0, 0, DT);
      constexpr uint32_t IDESC_G = idesc_f16_f32(BM, D, 0, 1, DT);
      auto q_tile = [&](int g) { return sbase + C::OFF_Q + (g % C::NST) * C::Q_TILE_BYTES; };
      auto do_tile = [&](int g) { return sbase + C::OFF_DO + (g % C::NST) * C::Q_TILE_BYTES; };
      SDesc kd = desc_k_base<D>(sbase + C::OFF_K);
      SDesc vd = desc_k_base<D>(sbase + C::OFF_V);
      auto issue_s = [&](int g) {  // S^T -> buffer g & 1
        const SDesc qd = desc_k_base<D>(q_tile(g));
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          umma_ss(tmem + (g & 1) * 128, sdesc_at(kd, k_major_off<D, BM>(ks)), sdesc_at(qd, k_major_off<D, BQ>(ks)),
                  IDESC_ST, ks > 0);
        umma_commit(s_full + (g & 1));
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
      // A operand (fp16 in TMEM) for query rows [16ks, 16ks+16) of a region
      // whose halves sit 64 columns apart
      auto a_col = [](int ks) { return uint32_t((ks >> 2) * 64 + (ks & 3) * 8); };
      int gi = 0, tcn = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int t = snake_unit(cta, k, n_cta, n_tiles);
        if (t >= n_tiles) break;
        const int n = tile_of<VL>(shp, t).n_items;
        if (n == 0) continue;
        const int kb = tcn & 1;
        if (!mbar_wait(kv_full + kb, uint32_t(tcn >> 1) & 1, ctl, 170)) { ok = false; break; }
        tc_fence_after();
        kd = desc_k_base<D>(sbase + C::OFF_K + kb * C::KV_TILE_BYTES);
        vd = desc_k_base<D>(sbase + C::OFF_V + kb * C::KV_TILE_BYTES);
        // the tile's first S^T and dP^T, and the second S^T, run while the
        // warpgroups finish the previous tile
        if (!wait_full(gi, 171)) { ok = false; break; }
        issue_s(gi);
        issue_dp(gi);
        if (n > 1) {
          if (!wait_full(gi + 1, 172)) { ok = false; break; }
          issue_s(gi + 1);
        }
        for (int it = 0; it < n; ++it) {
          const int g = gi + it;
          if (!mbar_wait(p_ready + (g & 1), uint32_t(g >> 1) & 1, ctl, 173)) { ok = false; break; }
          // dV / dK of the previous tile were read by the epilogue
          if (it == 0 && tcn > 0 && !mbar_wait(acc_empty, uint32_t(tcn - 1) & 1, ctl, 177)) { ok = false; break; }
          tc_fence_after();
          {
            const SDesc dd = desc_mn_base<D, BQ>(do_tile(g));
            const uint32_t pa = tmem + (g & 1) * 128;
            umma_ts(tmem + C::DV_COL, pa, sdesc_at(dd, 0), IDESC_G, it > 0 ? 1u : 0u);
#pragma unroll
            for (int ks = 1; ks < BQ / 16; ++ks)
              umma_ts(tmem + C::DV_COL, pa + a_col(ks), sdesc_at(dd, mn_major_off<D>(ks)), IDESC_G, 1u);
          }
          if (!mbar_wait(ds_ready, uint32_t(g) & 1, ctl, 174)) { ok = false; break; }
          tc_fence_after();
          {
            const SDesc qd = desc_mn_base<D, BQ>(q_tile(g));
            umma_ts(tmem + C::DK_COL, tmem + C::DP_COL, sdesc_at(qd, 0), IDESC_G, it > 0 ? 1u : 0u);
#pragma unroll
            for (int ks = 1; ks < BQ / 16; ++ks)
              umma_ts(tmem + C::DK_COL, tmem + C::DP_COL + a_col(ks), sdesc_at(qd, mn_major_off<D>(ks)), IDESC_G,
                      1u);
          }
          umma_commit(empty + g % C::NST);
          if (it + 1 < n) issue_dp(g + 1);  // its stage was waited for before S^T(g+1)
          // buffer g&1 is free: dV(g) (issued above) and warpgroup 1 (before
          // ds_ready) have read P^T(g)
          if (it + 2 < n) {
            if (!wait_full(g + 2, 175)) { ok = false; break; }
            issue_s(g + 2);
          }
        }
        if (!ok) break;
        umma_commit(acc_full);
        umma_commit(kv_empty + kb);
        gi += n;
        ++tcn;
      }
      umma_commit(mma_done);
      mbar_wait_drain(mma_done, 0, ctl, 176);
    }
  } else if (warp >= 4) {
    // =================== P^T (warpgroup 0) / dS^T (warpgroup 1) ===================
    const int w = (warp - 4) / 4;  // 0: exponentials, 1: dS^T
    const int wq = warp & 3;
    const int rl = wq * 32 + lane;  // key row within the tile
    const uint32_t lane_base = tmem_addr(tmem, uint32_t(wq * 32), 0);
    const uint64_t c2x2 = f2pack(shp.scale_log2, shp.scale_log2);
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
        if (w == 0 && wt.n_items > 0) mw_next = mask_words(0);
      }
      for (int it = 0; it < wt.n_items && ok; ++it) {
        const int g = gi + it;
        const int s = g % C::NST;
        const int q0 = (wt.i_start + it % wt.per_head) * BQ;
        if (w == 0) {
          uint4 mw;
          if constexpr (BITS) {
            mw = mw_next;
            if (it + 1 < wt.n_items) mw_next = mask_words(it + 1);
          }
          if (!mbar_wait_warp(s_full + (g & 1), uint32_t(g >> 1) & 1, ctl, 180)) { ok = false; break; }
          // the stage's -lse2/-Delta: its phase completed before S^T was issued
          if (!mbar_wait_warp(full + s, uint32_t(g / C::NST) & 1, ctl, 182)) { ok = false; break; }
          tc_fence_after();
#pragma unroll 1
          for (int hh = 0; hh < 2; ++hh) {
            const uint32_t tS = lane_base + uint32_t((g & 1) * 128 + 64 * hh);
            float st[64];
            tmem_ld64(tS, st);
            int cmin = key_out ? 64 : 0;
            if (shp.causal && !key_out) {
              const long long x = cmin_base - q0 - 64 * hh;
              cmin = x <= 0 ? 0 : (x > 64 ? 64 : int(x));
            }
            if (cmin > 0) {
#pragma unroll
              for (int c = 0; c < 64; ++c) st[c] = c >= cmin ? st[c] : -INFINITY;
            }
            if (VL && shp.window > 0 && !key_out) {
              // sliding window: queries past this key's window do not see it
              const long long xm = cmin_base + shp.window - 1 - q0 - 64 * hh;  // last visible column
              if (xm < 63) {
#pragma unroll
                for (int c = 0; c < 64; ++c) st[c] = c <= xm ? st[c] : -INFINITY;
              }
            }
            if constexpr (BITS) {
              const uint32_t words[2] = {hh ? mw.z : mw.x, hh ? mw.w : mw.y};
              if ((words[0] & words[1]) != 0xffffffffu) apply_mask_bits<64>(st, words);
            }
            const float4* l4 = reinterpret_cast<const float4*>(s_nlse + s * BQ + 64 * hh);
            uint32_t pk_p[32];
#pragma unroll
            for (int c4 = 0; c4 < 16; ++c4) {
              const float4 nl = l4[c4];
              const int c = c4 * 4;
              const uint64_t x01 = ffma2(f2pack(st[c], st[c + 1]), c2x2, f2pack(nl.x, nl.y));
              const uint64_t x23 = ffma2(f2pack(st[c + 2], st[c + 3]), c2x2, f2pack(nl.z, nl.w));
              const uint64_t e01 = ((2 * c4) & 7) < POLY_MASK ? exp2_poly2(x01) : exp2_mufu2(x01);
              const uint64_t e23 = ((2 * c4 + 1) & 7) < POLY_MASK ? exp2_poly2(x23) : exp2_mufu2(x23);
              pk_p[c4 * 2] = pack2_f2<DT>(e01);
              pk_p[c4 * 2 + 1] = pack2_f2<DT>(e23);
            }
            tmem_st16(tS, *reinterpret_cast<uint32_t(*)[16]>(&pk_p[0]));
            tmem_st16(tS + 16, *reinterpret_cast<uint32_t(*)[16]>(&pk_p[16]));
          }
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(p_ready + (g & 1));
        } else {
          if (!mbar_wait_warp(p_ready + (g & 1), uint32_t(g >> 1) & 1, ctl, 184)) { ok = false; break; }
          if (!mbar_wait_warp(dp_full, uint32_t(g) & 1, ctl, 185)) { ok = false; break; }
          if (!mbar_wait_warp(full + s, uint32_t(g / C::NST) & 1, ctl, 183)) { ok = false; break; }
          tc_fence_after();
#pragma unroll 1
          for (int hh = 0; hh < 2; ++hh) {
            const uint32_t tD = lane_base + uint32_t(C::DP_COL + 64 * hh);
            float dpt[64];
            tmem_ld64(tD, dpt);
            float pf[32];
            tmem_ld32(lane_base + uint32_t((g & 1) * 128 + 64 * hh), pf);
            const float4* d4 = reinterpret_cast<const float4*>(s_ndelta + s * BQ + 64 * hh);
            uint32_t pk_ds[32];
#pragma unroll
            for (int c4 = 0; c4 < 16; ++c4) {
              const float4 nd = d4[c4];
              const int c = c4 * 4;
              // dS = P (dP - Delta), P arriving packed from the P^T
              // warpgroup.  bf16: P widened (two shifts), the product in
              // fp32, one rounding.  fp16: the product in fp16 (widening an
              // fp16 P exactly costs integer work that made the kernel 8%
              // slower for a few percent less error, measured).
              const uint64_t d01f = fadd2(f2pack(dpt[c], dpt[c + 1]), f2pack(nd.x, nd.y));
              const uint64_t d23f = fadd2(f2pack(dpt[c + 2], dpt[c + 3]), f2pack(nd.z, nd.w));
              if constexpr (DT == DT_BF16) {
                pk_ds[c4 * 2] = pack2_f2<DT>(fmul2(widen_bf16x2(__float_as_uint(pf[c4 * 2])), d01f));
                pk_ds[c4 * 2 + 1] = pack2_f2<DT>(fmul2(widen_bf16x2(__float_as_uint(pf[c4 * 2 + 1])), d23f));
              } else {
                pk_ds[c4 * 2] = mul2<DT>(__float_as_uint(pf[c4 * 2]), pack2_f2<DT>(d01f));
                pk_ds[c4 * 2 + 1] = mul2<DT>(__float_as_uint(pf[c4 * 2 + 1]), pack2_f2<DT>(d23f));
              }
            }
            tmem_st16(tD, *reinterpret_cast<uint32_t(*)[16]>(&pk_ds[0]));
            tmem_st16(tD + 16, *reinterpret_cast<uint32_t(*)[16]>(&pk_ds[16]));
          }
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(ds_ready);
        }
      }
      if (!ok) break;
      // ---- epilogue of the tile: warpgroup 0 stores dV, warpgroup 1 stores dK ----
      if (wt.n_items > 0) {
        if (!mbar_wait_warp(acc_full, uint32_t(tcn) & 1, ctl, 186 + w)) { ok = false; break; }
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
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int D, int DT, bool VL, bool BITS = false>
int launch_bwd_dkdv_wide_t(const BwdArgs& a) {
  using C = bkvw::Cfg<D>;
  auto kern = fa_bwd_dkdv_wide_kernel<D, DT, VL, BITS>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) != cudaSuccess)
    return FA_ERR_LAUNCH;
  const int n_kt = (a.shape.Nk + bkvw::BM - 1) / bkvw::BM;
  const int n_tiles = n_kt * a.shape.B * a.shape.Hkv;
  const int sms = device_sm_count();
  const int n_cta = n_tiles < sms ? n_tiles : sms;
  kern<<<dim3(unsigned(n_cta)), bkvw::NUM_THREADS, C::SMEM_BYTES, a.stream>>>(
      a.tmap_q, a.tmap_do, a.tmap_k, a.tmap_v, a.shape, a.lse, a.delta, a.dk, a.dk_sb, a.dk_sh, a.dk_sn, a.dv, a.dv_sb,
      a.dv_sh, a.dv_sn, a.accumulate_fp32, n_tiles, a.mask);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

template <int D, int DT, bool VL, bool BITS = false, bool DROP = false>
int launch_bwd_dkdv_t(const BwdArgs& a) {
  using C = bkv::Cfg<D>;
  auto kern = fa_bwd_dkdv_kernel<D, DT, VL, BITS, DROP>;
  // The register split inside the kernel assumes the launch count; a build
  // that allocated a different number must not run (an increase that does
  // not fit would wait forever).
  static int regs_ok = -1;
  if (regs_ok < 0) {
    cudaFuncAttributes fa_attr;
    regs_ok = cudaFuncGetAttributes(&fa_attr, kern) == cudaSuccess && fa_attr.numRegs == int(bkv::LAUNCH_REGS) ? 1 : 0;
  }
  if (!regs_ok) return FA_ERR_LAUNCH;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) != cudaSuccess)
    return FA_ERR_LAUNCH;
  const int n_kt = (a.shape.Nk + bkv::BM - 1) / bkv::BM;
  const int n_tiles = n_kt * a.shape.B * a.shape.Hkv;
  const int sms = device_sm_count();
  const int n_cta = n_tiles < sms ? n_tiles : sms;
  kern<<<dim3(unsigned(n_cta)), bkv::NUM_THREADS, C::SMEM_BYTES, a.stream>>>(
      a.tmap_q, a.tmap_do, a.tmap_k, a.tmap_v, a.shape, a.lse, a.delta, a.dk, a.dk_sb, a.dk_sh, a.dk_sn, a.dv, a.dv_sb,
      a.dv_sh, a.dv_sn, a.accumulate_fp32, n_tiles, a.mask, a.drop);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

// Dense and packed (varlen) layouts are separate instantiations, so the
// dense kernels carry no per-batch offset arithmetic.
template <int D, int DT>
int launch_bwd_dkdv_l(const BwdArgs& a) {
  // dropout: every head size runs the kernel whose warpgroups build P^T and
  // dS^T of an item together in registers (dense layout, no mask)
  if (a.drop.t) return launch_bwd_dkdv_t<D, DT, false, false, true>(a);
  if constexpr (D == 128) {
    if (a.mask.bits) return launch_bwd_dkdv_t<D, DT, false, true>(a);  // dense layout only
    return a.shape.cu_q ? launch_bwd_dkdv_t<D, DT, true>(a) : launch_bwd_dkdv_t<D, DT, false>(a);
  } else {
    if (a.mask.bits) return launch_bwd_dkdv_wide_t<D, DT, false, true>(a);
    return a.shape.cu_q ? launch_bwd_dkdv_wide_t<D, DT, true>(a) : launch_bwd_dkdv_wide_t<D, DT, false>(a);
  }
}

int launch_bwd_dkdv(const BwdArgs& a, int D) {
  switch (D) {
    case 32: return a.dtype == DT_BF16 ? launch_bwd_dkdv_l<32, DT_BF16>(a) : launch_bwd_dkdv_l<32, DT_F16>(a);
    case 64: return a.dtype == DT_BF16 ? launch_bwd_dkdv_l<64, DT_BF16>(a) : launch_bwd_dkdv_l<64, DT_F16>(a);
    case 128: return a.dtype == DT_BF16 ? launch_bwd_dkdv_l<128, DT_BF16>(a) : launch_bwd_dkdv_l<128, DT_F16>(a);
    default: return FA_ERR_UNSUPPORTED_HEAD_DIM;
  }
}

}  // namespace fa
