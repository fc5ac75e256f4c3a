// fa_bwd_fused128.cu -- FlashAttention-2 backward in one pass over the key
// tiles at D = 128 for B200 (sm_100a).
//
// Produces what the reference's _attn_bwd produces at head dim 128
// (triton_flash_attention/attention.py:383-573, _SUPPORTED_HEAD_DIMS at :21):
// dK and dV as its dK/dV half (:428-505, inner loop :259-308) and dQ as its
// dQ half (:507-573, inner loop :312-350), in one visit of every (key tile,
// query tile) pair instead of the reference's two recomputations of P and
// dS -- the GEMM work is the 2.5x forward that the metric credits, where the
// separate dQ and dK/dV kernels execute 3.5x:
//   P^T = exp2(scale*log2(e) * K Q^T - lse2),  dP^T = V dO^T,
//   dS^T = P^T (dP^T - Delta),
//   dV += P^T dO,  dK += dS^T Q          (in TMEM for the whole key tile),
//   dQ^T_part = K^T dS^T                 (one D x 64 partial per item),
// and each dQ partial is added into an fp32 accumulator [B, Hq, Nq, 128] by
// TMA reduce-add, scaled by the softmax scale.  dQ is therefore not bitwise
// reproducible run to run (its fp32 additions follow the schedule); dK, dV
// are (one CTA owns a key tile and sums the group's query heads itself).
//
// Why dQ^T: at D = 128 the dK and dV accumulators take 256 of the 512 TMEM
// columns and each 64-query item needs S^T and dP^T (64 columns each, two
// items in flight), which leaves no 128-column slot for a 64 x 128 dQ
// partial.  K^T dS^T puts D on the TMEM lanes and the item's 64 queries on
// 64 columns -- exactly the dP^T columns, free once the item's dS^T has been
// read by the dK MMA (tcgen05.mma runs in issue order).  Its operands are
// the resident K tile read as an MN-major A (M = D) and the item's dS^T tile
// in shared memory read as an MN-major B (N = queries): no transpose is
// materialised anywhere.
//
// Work layout: a persistent CTA per SM walks work tiles of 128 keys of one
// (batch, kv head) in snake order (fa_key_tiles.cuh); an item is one (query
// head of the group, 64-row query tile).  Warp roles (512 threads):
//  * warp 0: TMA of K and the Q tiles, plain loads of lse2 / Delta;
//  * warp 3: TMA of V and the dO tiles (in both, lanes 0 and 1 issue a
//    tile's two 64-column boxes);
//  * warp 1: one thread issues every tcgen05.mma;
//  * warp 2: owns the TMEM allocation;
//  * warps 4-7 / 8-11: the elementwise warpgroups, items of even / odd
//    index, one thread per key row: P^T and dS^T (fp16 / bf16) back into
//    TMEM for the dV and dK MMAs, and dS^T into the warpgroup's shared-memory
//    tile (128-byte swizzle) for the dQ^T MMA;
//  * warps 12-15: read the dQ^T partial from TMEM (thread = head-dim
//    column, 64 queries), scale it, stage it in shared memory (each warp its
//    32 columns x 64 rows) and issue that warp's TMA reduce-add, so four
//    threads feed the TMA unit.
// TMEM (512 columns): item buffer b = g & 1 at [128b, 128b+128): S^T at +0
//   (P^T packed into +0..32 once read), dP^T at +64 (dS^T packed into
//   +64..96, then the item's dQ^T at +64..128); dV at [256,384), dK at
//   [384,512).
// Shared memory (227 KB): K and V tiles (one buffer each: a tile's items
// far outnumber the start-up its reload costs), Q/dO in 3 stages, two dS^T
// tiles, four 8 KB dQ staging pieces.
#include "fa_common.cuh"
#include "fa_kernels.h"
#include "fa_key_tiles.cuh"

namespace fa {

namespace bf128 {
constexpr int D = 128;
constexpr int BM = 128;  // keys per tile
constexpr int BQ = 64;   // query rows per item
constexpr int NUM_THREADS = 512;
// Registers per thread: launched at 128 (512 threads); warps 0-3 drop to
// CTRL_REGS and the dQ warpgroup to DQ_REGS, the two elementwise warpgroups
// rise to SOFT_REGS.  The shares must add up to at most 512 * 128 = 65536.
constexpr uint32_t LAUNCH_REGS = 128;
constexpr uint32_t CTRL_REGS = 96;
constexpr uint32_t DQ_REGS = 96;
constexpr uint32_t SOFT_REGS = 160;
static_assert(128 * CTRL_REGS + 128 * DQ_REGS + 256 * SOFT_REGS <= NUM_THREADS * LAUNCH_REGS, "register split");

struct Cfg {
  using G = TileGeom<D>;
  static constexpr int NST = 3;
  static constexpr int KV_TILE_BYTES = BM * D * 2;
  static constexpr int Q_TILE_BYTES = BQ * D * 2;
  static constexpr int DS_BYTES = BM * BQ * 2;        // 128 key rows x 64 queries (128 B rows)
  static constexpr int DQ_PIECE_BYTES = BQ * 32 * 4;  // one warp's 32 fp32 columns x 64 rows
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + KV_TILE_BYTES;
  static constexpr int OFF_Q = OFF_V + KV_TILE_BYTES;
  static constexpr int OFF_DO = OFF_Q + NST * Q_TILE_BYTES;
  static constexpr int OFF_DS = OFF_DO + NST * Q_TILE_BYTES;  // one tile per item parity
  static constexpr int OFF_DQS = OFF_DS + 2 * DS_BYTES;        // one piece per dQ warp
  static constexpr int OFF_LSE = OFF_DQS + 4 * DQ_PIECE_BYTES;
  static constexpr int OFF_DELTA = OFF_LSE + NST * BQ * 4;
  static constexpr int OFF_BAR = OFF_DELTA + NST * BQ * 4;
  // kv_full, kv_empty, full[NST], empty[NST], st_full[2], ds_ready[2], ds_free[2], dq_full[2], dq_empty[2],
  // acc_full, acc_empty, mma_done
  static constexpr int NUM_BARS = 2 + 2 * NST + 5 * 2 + 3;
  static constexpr int OFF_CTL = OFF_BAR + NUM_BARS * 8;
  static constexpr int OFF_MISC = OFF_CTL + 16;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr int DP_COL = 64;  // within an item buffer
  static constexpr int DV_COL = 256;
  static constexpr int DK_COL = 384;
  static_assert(DK_COL + D <= TMEM_COLS, "TMEM budget");
  static_assert(OFF_DS % 1024 == 0 && OFF_Q % 1024 == 0 && OFF_DO % 1024 == 0, "swizzled tiles need 1024-byte alignment");
  static_assert(OFF_DQS % 128 == 0, "TMA source alignment");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

using Tile = KeyTile;
template <bool VL>
__device__ __forceinline__ Tile tile_of(const AttnShape& shp, int t) {
  return key_tile_of<VL, BM, BQ>(shp, t);
}
template <bool VL>
using ItemCursor = KeyItemCursor<VL, BM, BQ>;
}  // namespace bf128

template <int DT, bool VL>
__global__ void __launch_bounds__(bf128::NUM_THREADS, 1)
    fa_bwd_fused128_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_do,
                           const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                           const __grid_constant__ CUtensorMap tmap_dq, const AttnShape shp,
                           const float* __restrict__ lse, const float* __restrict__ delta, void* __restrict__ dk_out,
                           const long long dk_sb, const long long dk_sh, const long long dk_sn,
                           void* __restrict__ dv_out, const long long dv_sb, const long long dv_sh,
                           const long long dv_sn, const int accumulate_fp32, const int n_tiles) {
  using namespace bf128;
  using C = Cfg;
  using G = TileGeom<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_saddr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_saddr + 1023u) & ~1023u) - raw_saddr);
  const uint32_t sbase = smem_u32(smem);

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* kv_full = bars;             // one phase per non-empty tile: K and V landed
  uint64_t* kv_empty = kv_full + 1;     // one phase per non-empty tile: its MMAs completed
  uint64_t* full = kv_empty + 1;
  uint64_t* empty = full + C::NST;
  // Per item parity b (phase k of barrier b belongs to item 2k + b, items
  // counted across the CTA's tiles):
  uint64_t* st_full = empty + C::NST;  // S^T, dP^T in TMEM
  uint64_t* ds_ready = st_full + 2;    // P^T, dS^T in TMEM and dS^T in shared memory
  uint64_t* ds_free = ds_ready + 2;    // the dQ^T MMA read the dS^T tile
  uint64_t* dq_full = ds_free + 2;     // dQ^T in TMEM
  uint64_t* dq_empty = dq_full + 2;    // the dQ warpgroup read dQ^T
  uint64_t* acc_full = dq_empty + 2;   // one phase per non-empty tile: dV, dK complete
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
    mbar_init(kv_full, 2);  // K from warp 0, V from warp 3
    mbar_init(kv_empty, 1);
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(full + s, 2 + 32);  // two TMA expect_tx arrives + one arrive per lane of warp 0
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(st_full + b, 1);
      mbar_init(ds_ready + b, 128);
      mbar_init(ds_free + b, 1);
      mbar_init(dq_full + b, 1);
      mbar_init(dq_empty + b, 128);
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
      const bool is_q = warp == 0;
      const CUtensorMap* tmap_kv = is_q ? &tmap_k : &tmap_v;
      const CUtensorMap* tmap_qd = is_q ? &tmap_q : &tmap_do;
      const int kv_off = is_q ? C::OFF_K : C::OFF_V;
      const int qd_off = is_q ? C::OFF_Q : C::OFF_DO;
      if (lane == 0) {
        tma_prefetch_desc(tmap_qd);
        tma_prefetch_desc(tmap_kv);
      }
      // lse2 / Delta of an item's 64 query rows (two per lane) are read with
      // plain loads issued PF items ahead, across tile boundaries.  Rows past
      // Nq, or rows that see no key, get lse2 = +inf so that their P is 0.
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
        // one K/V buffer: the previous tile's MMAs have completed
        if (tcn >= 1 && !mbar_wait_warp(kv_empty, uint32_t(tcn - 1) & 1, ctl, 300)) {
          ok = false;
          break;
        }
        // the tile's two 64-column boxes come from two lanes: one thread's
        // TMA loads are processed one after another (C4: -5 %, measured)
        if (lane == 0) mbar_arrive_expect_tx(kv_full, C::KV_TILE_BYTES);
        __syncwarp();
        if (lane < G::NBOX)
          tma_load_4d(smem + kv_off + lane * BM * G::SW, tmap_kv, kv_full, lane * G::BOX, w.sq.k0 + w.kv0, w.kvh,
                      w.sq.tb);
        ++tcn;
        for (int it = 0; it < w.n_items; ++it) {
          if (is_q) fetch(lv[PF], dvv[PF]);
          const int s = gi % C::NST;
          const uint32_t u = uint32_t(gi / C::NST);
          if (u > 0 && !mbar_wait_warp(empty + s, (u - 1) & 1, ctl, 301)) {
            ok = false;
            break;
          }
          const int h = w.kvh * group + it / w.per_head;
          const int q0 = (w.i_start + it % w.per_head) * BQ;
          if (lane == 0) mbar_arrive_expect_tx(full + s, C::Q_TILE_BYTES);
          __syncwarp();
          if (lane < G::NBOX)
            tma_load_4d(smem + qd_off + s * C::Q_TILE_BYTES + lane * BQ * G::SW, tmap_qd, full + s, lane * G::BOX,
                        w.sq.q0 + q0, h, w.sq.tb);
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
        if (tcn > 0) mbar_wait_drain(kv_full, uint32_t(tcn - 1) & 1, ctl, 302);
        for (int j = (gi > C::NST ? gi - C::NST : 0); j < gi; ++j)
          mbar_wait_drain(full + j % C::NST, uint32_t(j / C::NST) & 1, ctl, 303);
      }
    } else if (warp == 1) {
      // =================== tcgen05 MMA issuer ===================
      if (lane == 0) {
        constexpr uint32_t IDESC_ST = idesc_f16_f32(BM, BQ, 0, 0, DT);  // S^T, dP^T: K-major A and B
        constexpr uint32_t IDESC_G = idesc_f16_f32(BM, D, 0, 1, DT);    // dV, dK: A in TMEM, MN-major B
        constexpr uint32_t IDESC_DQ = idesc_f16_f32(D, BQ, 1, 1, DT);   // dQ^T: MN-major A (K^T) and B (dS^T)
        auto q_tile = [&](int g) { return sbase + C::OFF_Q + (g % C::NST) * C::Q_TILE_BYTES; };
        auto do_tile = [&](int g) { return sbase + C::OFF_DO + (g % C::NST) * C::Q_TILE_BYTES; };
        const SDesc kd = desc_k_base<D>(sbase + C::OFF_K);
        const SDesc vd = desc_k_base<D>(sbase + C::OFF_V);
        // K^T as the A operand of dQ^T: M = 128 head-dim columns in two
        // 64-column boxes (LBO apart), K = 128 keys (rows of 128 bytes)
        const SDesc kmn = desc_mn_base<D, BM>(sbase + C::OFF_K);
        bool ok = true;
        auto wait_full = [&](int g, int site) {
          const bool r = mbar_wait(full + g % C::NST, uint32_t(g / C::NST) & 1, ctl, site);
          tc_fence_after();
          return r;
        };
        // S^T(g), dP^T(g) -> item buffer g & 1; dP^T overwrites dQ^T(g - 2),
        // so it waits until the dQ warpgroup read that
        auto issue_st = [&](int g) {
          const uint32_t buf = tmem + uint32_t(g & 1) * 128;
          if (!wait_full(g, 310)) return false;
          const SDesc qd = desc_k_base<D>(q_tile(g));
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
            umma_ss(buf, sdesc_at(kd, k_major_off<D, BM>(ks)), sdesc_at(qd, k_major_off<D, BQ>(ks)), IDESC_ST, ks > 0);
          if (g >= 2 && !mbar_wait(dq_empty + (g & 1), uint32_t((g - 2) >> 1) & 1, ctl, 311)) return false;
          tc_fence_after();
          const SDesc dd = desc_k_base<D>(do_tile(g));
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
            umma_ss(buf + C::DP_COL, sdesc_at(vd, k_major_off<D, BM>(ks)), sdesc_at(dd, k_major_off<D, BQ>(ks)),
                    IDESC_ST, ks > 0);
          umma_commit(st_full + (g & 1));
          return true;
        };
        int gi = 0, tcn = 0;
        for (int k = 0; ok; ++k) {
          const int t = snake_unit(cta, k, n_cta, n_tiles);
          if (t >= n_tiles) break;
          const int n = tile_of<VL>(shp, t).n_items;
          if (n == 0) continue;
          if (!mbar_wait(kv_full, uint32_t(tcn) & 1, ctl, 312)) { ok = false; break; }
          tc_fence_after();
          if (!issue_st(gi)) { ok = false; break; }
          if (n > 1 && !issue_st(gi + 1)) { ok = false; break; }
          for (int it = 0; it < n; ++it) {
            const int g = gi + it;
            const int b = g & 1;
            const uint32_t buf = tmem + uint32_t(b) * 128;
            if (!mbar_wait(ds_ready + b, uint32_t(g >> 1) & 1, ctl, 313)) { ok = false; break; }
            // dV / dK of the previous tile were read by the epilogue
            if (it == 0 && tcn > 0 && !mbar_wait(acc_empty, uint32_t(tcn - 1) & 1, ctl, 314)) { ok = false; break; }
            tc_fence_after();
            const uint32_t acc = (it > 0) ? 1u : 0u;
            {  // dV += P^T dO: A = P^T packed in the buffer's columns [0, 32)
              const SDesc dd = desc_mn_base<D, BQ>(do_tile(g));
              umma_ts(tmem + C::DV_COL, buf, sdesc_at(dd, 0), IDESC_G, acc);
#pragma unroll
              for (int ks = 1; ks < BQ / 16; ++ks)
                umma_ts(tmem + C::DV_COL, buf + ks * 8, sdesc_at(dd, mn_major_off<D>(ks)), IDESC_G, 1u);
            }
            {  // dK += dS^T Q: A = dS^T packed in columns [64, 96)
              const SDesc qd = desc_mn_base<D, BQ>(q_tile(g));
              umma_ts(tmem + C::DK_COL, buf + C::DP_COL, sdesc_at(qd, 0), IDESC_G, acc);
#pragma unroll
              for (int ks = 1; ks < BQ / 16; ++ks)
                umma_ts(tmem + C::DK_COL, buf + C::DP_COL + ks * 8, sdesc_at(qd, mn_major_off<D>(ks)), IDESC_G, 1u);
            }
            umma_commit(empty + g % C::NST);  // the item's Q / dO stage is consumed
            {  // dQ^T = K^T dS^T into columns [64, 128), over dS^T that dK has read
              const SDesc dsd = desc_mn_base<BQ, BM>(sbase + C::OFF_DS + b * C::DS_BYTES);
#pragma unroll
              for (int ks = 0; ks < BM / 16; ++ks)
                umma_ss(buf + C::DP_COL, sdesc_at(kmn, mn_major_off<D>(ks)), sdesc_at(dsd, mn_major_off<BQ>(ks)),
                        IDESC_DQ, ks > 0);
              umma_commit(dq_full + b);
              umma_commit(ds_free + b);
            }
            if (it + 2 < n && !issue_st(g + 2)) { ok = false; break; }
          }
          if (!ok) break;
          umma_commit(acc_full);
          umma_commit(kv_empty);
          gi += n;
          ++tcn;
        }
        umma_commit(mma_done);
        mbar_wait_drain(mma_done, 0, ctl, 315);
      }
    }
  } else if (warp < 12) {
    regs_claim<SOFT_REGS>();
    // =================== P^T / dS^T warpgroups ===================
    const int w = (warp - 4) / 4;  // item parity of this warpgroup
    const int wq = warp & 3;
    const int rl = wq * 32 + lane;  // key row within the tile
    const uint32_t tB = tmem_addr(tmem, uint32_t(wq * 32), uint32_t(w * 128));
    const uint64_t c2x2 = f2pack(shp.scale_log2, shp.scale_log2);
    // this thread's row of the warpgroup's swizzled dS^T tile
    const uint32_t ds_row = sbase + C::OFF_DS + uint32_t(w * C::DS_BYTES) + uint32_t(rl) * 128u;
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
      for (int it = (gi & 1) == w ? 0 : 1; it < wt.n_items; it += 2) {
        const int g = gi + it;
        const int s = g % C::NST;
        const int q0 = (wt.i_start + it % wt.per_head) * BQ;
        if (!mbar_wait_warp(st_full + w, uint32_t(g >> 1) & 1, ctl, 320 + w)) { ok = false; break; }
        // the stage's -lse2 / -Delta: its phase completed before S^T was issued
        if (!mbar_wait_warp(full + s, uint32_t(g / C::NST) & 1, ctl, 322 + w)) { ok = false; break; }
        tc_fence_after();
        int cmin = key_out ? BQ : 0;
        if (shp.causal && !key_out) {
          const long long x = cmin_base - q0;
          cmin = x <= 0 ? 0 : (x > BQ ? BQ : int(x));
        }
        long long xm = BQ;  // sliding window: last visible query column
        if (VL && shp.window > 0 && !key_out) xm = cmin_base + shp.window - 1 - q0;
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
          float st[32], dpt[32];
          tmem_ld32(tB + uint32_t(32 * hh), st);
          tmem_ld32(tB + uint32_t(C::DP_COL + 32 * hh), dpt);
          const int cm = cmin - 32 * hh;
          if (cm > 0) {  // causal diagonal: queries before this key are invisible
#pragma unroll
            for (int c = 0; c < 32; ++c) st[c] = c >= cm ? st[c] : -INFINITY;
          }
          if (VL && xm - 32 * hh < 31) {
            const long long xh = xm - 32 * hh;
#pragma unroll
            for (int c = 0; c < 32; ++c) st[c] = c <= xh ? st[c] : -INFINITY;
          }
          // stage values are stored negated: -lse2 and -Delta
          const float4* l4 = reinterpret_cast<const float4*>(s_nlse + s * BQ + 32 * hh);
          const float4* d4 = reinterpret_cast<const float4*>(s_ndelta + s * BQ + 32 * hh);
          uint32_t pk_p[16], pk_ds[16];
#pragma unroll
          for (int c4 = 0; c4 < 8; ++c4) {
            const float4 nl = l4[c4];
            const float4 nd = d4[c4];
            const int c = c4 * 4;
            // dS = P (dP - Delta) in fp32, rounded once (as the reference's
            // dsT = pT * (dpT - Di) before .to(float16), attention.py:300-305)
            const uint64_t e01 = exp2_mufu2(ffma2(f2pack(st[c], st[c + 1]), c2x2, f2pack(nl.x, nl.y)));
            const uint64_t e23 = exp2_mufu2(ffma2(f2pack(st[c + 2], st[c + 3]), c2x2, f2pack(nl.z, nl.w)));
            pk_p[c4 * 2] = pack2_f2<DT>(e01);
            pk_p[c4 * 2 + 1] = pack2_f2<DT>(e23);
            pk_ds[c4 * 2] = pack2_f2<DT>(fmul2(e01, fadd2(f2pack(dpt[c], dpt[c + 1]), f2pack(nd.x, nd.y))));
            pk_ds[c4 * 2 + 1] = pack2_f2<DT>(fmul2(e23, fadd2(f2pack(dpt[c + 2], dpt[c + 3]), f2pack(nd.z, nd.w))));
          }
          // packed halves land on columns this thread has already read
          tmem_st16(tB + uint32_t(16 * hh), pk_p);
          tmem_st16(tB + uint32_t(C::DP_COL + 16 * hh), pk_ds);
          // the dQ^T MMA of this warpgroup's previous item has read the tile
          if (hh == 0 && g >= 2 && !mbar_wait_warp(ds_free + w, uint32_t((g - 2) >> 1) & 1, ctl, 324 + w)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int c = 0; c < 4; ++c)
            st_shared_v4(ds_row + ((uint32_t(4 * hh + c) ^ ds_swz) << 4), pk_ds[4 * c], pk_ds[4 * c + 1],
                         pk_ds[4 * c + 2], pk_ds[4 * c + 3]);
        }
        if (!ok) break;
        tmem_st_wait();
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(ds_ready + w);
      }
      if (!ok) break;
      // ---- epilogue of the tile: warpgroup 0 stores dV, warpgroup 1 stores dK ----
      if (wt.n_items > 0) {
        if (!mbar_wait_warp(acc_full, uint32_t(tcn) & 1, ctl, 326 + w)) { ok = false; break; }
        tc_fence_after();
      }
      const int kr = wt.kv0 + rl;
      const bool row_ok = kr < wt.sq.nk;
      const float sc = w == 0 ? 1.f : shp.scale;
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
  } else {
    regs_release<DQ_REGS>();
    // =================== dQ warpgroup ===================
    // Warp wq reads TMEM lanes [32 wq, 32 wq + 32): head-dim columns
    // d = 32 wq + lane of the item's 64 query rows.  Its staging piece is
    // [64 rows][32 fp32] without swizzle: for a fixed row the warp's 32
    // lanes write one contiguous 128-byte line.
    const int wq = warp & 3;
    const uint32_t lane_base = tmem_addr(tmem, uint32_t(wq * 32), 0);
    uint8_t* const piece = smem + C::OFF_DQS + wq * C::DQ_PIECE_BYTES;
    const uint32_t piece_lane = sbase + uint32_t(C::OFF_DQS + wq * C::DQ_PIECE_BYTES) + uint32_t(lane) * 4u;
    const float sc = shp.scale;
    int gi = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int t = snake_unit(cta, k, n_cta, n_tiles);
      if (t >= n_tiles) break;
      const Tile wt = tile_of<VL>(shp, t);
      for (int it = 0; it < wt.n_items; ++it) {
        const int g = gi + it;
        const int b = g & 1;
        const int h = wt.kvh * group + it / wt.per_head;
        const int q0 = (wt.i_start + it % wt.per_head) * BQ;
        if (!mbar_wait_warp(dq_full + b, uint32_t(g >> 1) & 1, ctl, 330)) { ok = false; break; }
        tc_fence_after();
        float acc[BQ];
        tmem_ld64(lane_base + uint32_t(b * 128 + C::DP_COL), acc);
        tc_fence_before();
        mbar_arrive(dq_empty + b);
        // this warp's previous reduce-add has finished reading the piece
        if (lane == 0 && g > 0) bulk_wait_read_all();
        __syncwarp();
#pragma unroll
        for (int r = 0; r < BQ; ++r)
          asm volatile("st.shared.f32 [%0], %1;" ::"r"(piece_lane + uint32_t(r) * 128u), "f"(acc[r] * sc) : "memory");
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_4d(&tmap_dq, piece, wq * 32, wt.sq.q0 + q0, h, wt.sq.tb);
          bulk_commit_group();
        }
      }
      if (!ok) break;
      gi += wt.n_items;
    }
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int DT, bool VL>
int launch_bwd_fused128_t(const BwdArgs& a, const CUtensorMap& tmap_dq) {
  using C = bf128::Cfg;
  auto kern = fa_bwd_fused128_kernel<DT, VL>;
  // The register split inside the kernel assumes the launch count; a build
  // that allocated a different number must not run (an increase that does
  // not fit would wait forever).
  static int regs_ok = -1;
  if (regs_ok < 0) {
    cudaFuncAttributes fa_attr;
    regs_ok = cudaFuncGetAttributes(&fa_attr, kern) == cudaSuccess && fa_attr.numRegs == int(bf128::LAUNCH_REGS) ? 1 : 0;
  }
  if (!regs_ok) return FA_ERR_LAUNCH;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) != cudaSuccess)
    return FA_ERR_LAUNCH;
  const int n_kt = (a.shape.Nk + bf128::BM - 1) / bf128::BM;
  const int n_tiles = n_kt * a.shape.B * a.shape.Hkv;
  const int sms = device_sm_count();
  const int n_cta = n_tiles < sms ? n_tiles : sms;
  kern<<<dim3(unsigned(n_cta)), bf128::NUM_THREADS, C::SMEM_BYTES, a.stream>>>(
      a.tmap_q, a.tmap_do, a.tmap_k, a.tmap_v, tmap_dq, a.shape, a.lse, a.delta, a.dk, a.dk_sb, a.dk_sh, a.dk_sn,
      a.dv, a.dv_sb, a.dv_sh, a.dv_sn, a.accumulate_fp32, n_tiles);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

// Dense and packed (varlen) layouts are separate instantiations; boolean
// masks and dropout at D = 128 run the separate dQ and dK/dV kernels.
int launch_bwd_fused128(const BwdArgs& a, const CUtensorMap& tmap_dq) {
  if (a.mask.bits || a.drop.t) return FA_ERR_UNSUPPORTED_HEAD_DIM;
  if (a.dtype == DT_BF16)
    return a.shape.cu_q ? launch_bwd_fused128_t<DT_BF16, true>(a, tmap_dq) : launch_bwd_fused128_t<DT_BF16, false>(a, tmap_dq);
  return a.shape.cu_q ? launch_bwd_fused128_t<DT_F16, true>(a, tmap_dq) : launch_bwd_fused128_t<DT_F16, false>(a, tmap_dq);
}

}  // namespace fa
