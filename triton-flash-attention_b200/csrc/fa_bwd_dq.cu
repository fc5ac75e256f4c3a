// fa_bwd_dq.cu -- FlashAttention-2 backward, dQ half, for B200 (sm_100a).
//
// Computes what the dQ half of the reference's _attn_bwd produces
// (triton_flash_attention/attention.py:507-573, inner loop :311-350):
//   P = exp2(scale*log2(e) * Q K^T - lse2),  dP = dO V^T,
//   dS = P (dP - Delta),  dQ = scale * dS K.
// Layout of the work (one persistent kernel for every head dim):
//  * a work tile is 128 query rows of one (batch, head); one CTA per SM walks
//    its share of the tiles and sweeps the 128-key tiles visible to each;
//  * warps 0 and 3 stream Q/dO and K/V through shared-memory stages with TMA;
//  * warp 1 (one thread) issues tcgen05.mma: S = Q K^T and dP = dO V^T into
//    TMEM, then dQ += dS K with dS read from TMEM (fp16/bf16, aliasing S) and
//    K read as an MN-major operand of the same shared tile;
//  * warps 4-7 / 8-11 turn S, dP into dS for key columns [0,64) / [64,128),
//    one thread per query row, with that row's lse2 and Delta in registers.
#include "fa_common.cuh"
#include "fa_kernels.h"

namespace fa {

// ---------------------------------------------------------------------------
// Persistent kernel with 128-key tiles, used for every D.  S = Q K^T and
// dP = dO V^T become N = 128 MMAs (full tensor rate; N = 64 runs at ~70%).
// One CTA per SM walks its share of the work tiles (128 query rows of one
// batch and head) back to back.  At D <= 64, Q and dO are double-buffered so
// that the next tile's loads and first MMAs overlap the current tile's last
// key tiles and its epilogue; at D = 128 shared memory holds one Q/dO buffer
// and two K/V stages.
// Both warpgroups work on every key tile, warpgroup w on key columns
// [64w, 64w+64), and S is double-buffered in TMEM so the tensor core computes
// S of tile j+2 and dP of tile j+1 while the warpgroups exponentiate tile j+1.
// TMEM: S buffers [0,128) and [128,256), dP [256,384), dQ [384, 384+D).
// Warpgroup w writes dS into its S buffer's columns [64w, 64w+32), inside the
// range it read.
namespace bdqw {
constexpr int BM = dq_cfg::BM;  // query rows per tile
constexpr int BN = dq_cfg::BN;  // keys per key tile
constexpr int NUM_THREADS = 384;
constexpr int POLY_MASK = 2;  // pairs (i & 7) < 2 use the FMA-pipe exp2: a quarter off MUFU

template <int D>
struct Cfg {
  using G = TileGeom<D>;
  static constexpr int NST = D == 128 ? 2 : 4;
  static constexpr int QB = D == 128 ? 1 : 2;  // Q/dO buffers (tiles in flight)
  static constexpr int Q_TILE_BYTES = BM * D * 2;
  static constexpr int KV_TILE_BYTES = BN * D * 2;
  static constexpr int OFF_Q = 0;                              // QB buffers
  static constexpr int OFF_DO = OFF_Q + QB * Q_TILE_BYTES;     // QB buffers
  static constexpr int OFF_K = OFF_DO + QB * Q_TILE_BYTES;     // NST stages
  static constexpr int OFF_V = OFF_K + NST * KV_TILE_BYTES;    // NST stages
  static constexpr int OFF_BAR = OFF_V + NST * KV_TILE_BYTES;
  // q_full[2], q_empty[2], kv_full[NST], kv_empty[NST], s_full[2], dp_full, ds_ready[2], dq_full, dq_empty, mma_done
  static constexpr int NUM_BARS = 2 + 2 + 2 * NST + 2 + 1 + 2 + 1 + 1 + 1;
  static constexpr int OFF_CTL = OFF_BAR + NUM_BARS * 8;
  static constexpr int OFF_MISC = OFF_CTL + 16;
  static constexpr int SMEM_USED = OFF_MISC + 16 + 1024;
  static constexpr int SMEM_BYTES = SMEM_USED;
  static constexpr int TMEM_COLS = 512;
  static constexpr int DP_COL = 256;
  static constexpr int DQ_COL = 384;
  static_assert(DQ_COL + D <= TMEM_COLS, "TMEM budget");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

// A work tile: 128 query rows of one (batch, query head) and the key tiles
// they see.  Tiles are numbered late query tiles first (the heavy ones under
// a causal mask).
struct Tile {
  int b, h, kvh, row0, kt0, n_kv;  // key tiles kt0 .. kt0 + n_kv - 1
  Seq sq;
};
template <bool WIN>
__device__ __forceinline__ Tile tile_of(const AttnShape& shp, int t) {
  const int BH = shp.B * shp.Hq;
  const int n_qt = (shp.Nq + BM - 1) / BM;
  Tile w;
  const int bh = t % BH;
  w.b = bh / shp.Hq;
  w.h = bh % shp.Hq;
  w.kvh = w.h / (shp.Hq / shp.Hkv);
  w.row0 = (n_qt - 1 - t / BH) * BM;
  w.sq = seq_of(shp, w.b);
  const int end = kv_tiles_for_rows(shp, w.sq, w.row0, BM, BN);
  const int first = WIN ? kv_first_tile(shp, w.sq, w.row0, BN) : 0;  // > 0 only under a sliding window
  w.kt0 = first < end ? first : 0;
  w.n_kv = first < end ? end - first : 0;
  return w;
}
}  // namespace bdqw

template <int D, int DT, bool WIN, bool BITS, bool DROP>
__global__ void __launch_bounds__(bdqw::NUM_THREADS, 1)
    fa_bwd_dq_wide_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_do,
                          const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                          const AttnShape shp, const float* __restrict__ lse, const float* __restrict__ delta,
                          void* __restrict__ dq_out, const long long dq_sb, const long long dq_sh,
                          const long long dq_sn, const int accumulate_fp32, const int n_tiles,
                          const MaskBits mk, const DropArgs dr) {
  using namespace bdqw;
  using C = Cfg<D>;
  using G = TileGeom<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_saddr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_saddr + 1023u) & ~1023u) - raw_saddr);
  const uint32_t sbase = smem_u32(smem);

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars;          // per Q/dO buffer
  uint64_t* q_empty = q_full + 2;   // per Q/dO buffer
  uint64_t* kv_full = q_empty + 2;
  uint64_t* kv_empty = kv_full + C::NST;
  uint64_t* s_full = kv_empty + C::NST;
  uint64_t* dp_full = s_full + 2;
  uint64_t* ds_ready = dp_full + 1;  // per S buffer
  uint64_t* dq_full = ds_ready + 2;  // one phase per non-empty tile
  uint64_t* dq_empty = dq_full + 1;  // one phase per non-empty tile: the epilogue read dQ
  uint64_t* mma_done = dq_empty + 1;
  CtaCtl* ctl_w = reinterpret_cast<CtaCtl*>(smem + C::OFF_CTL);
  volatile CtaCtl* ctl = ctl_w;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);

  const int warp = int(warp_id());
  const int lane = int(lane_id());
  const int cta = int(blockIdx.x);
  const int n_cta = int(gridDim.x);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(q_full + i, 2);
      mbar_init(q_empty + i, 1);
    }
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(kv_full + s, 2);
      mbar_init(kv_empty + s, 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_full + 1, 1);
    mbar_init(dp_full, 1);
    mbar_init(ds_ready, 256);
    mbar_init(ds_ready + 1, 256);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 256);
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
    // =================== TMA producers ===================
    // Warp 0 loads Q and the K tiles, warp 3 dO and the V tiles (one thread's
    // TMA loads are processed one after another); q_full and kv_full expect
    // one arrival from each.
    const bool is_k = warp == 0;
    if (lane == 0) {
      const CUtensorMap* tmap_kv = is_k ? &tmap_k : &tmap_v;
      const CUtensorMap* tmap_qd = is_k ? &tmap_q : &tmap_do;
      const int kv_off = is_k ? C::OFF_K : C::OFF_V;
      const int qd_off = is_k ? C::OFF_Q : C::OFF_DO;
      tma_prefetch_desc(tmap_qd);
      tma_prefetch_desc(tmap_kv);
      int gj = 0, tcn = 0;  // key tiles and non-empty tiles issued
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int t = snake_unit(cta, k, n_cta, n_tiles);
        if (t >= n_tiles) break;
        const Tile w = tile_of<WIN>(shp, t);
        if (w.n_kv == 0) continue;
        const int tb = tcn % C::QB;
        if (tcn >= C::QB && !mbar_wait(q_empty + tb, uint32_t(tcn / C::QB - 1) & 1, ctl, 130)) break;
        mbar_arrive_expect_tx(q_full + tb, C::Q_TILE_BYTES);
        for (int bx = 0; bx < G::NBOX; ++bx)
          tma_load_4d(smem + qd_off + tb * C::Q_TILE_BYTES + bx * BM * G::SW, tmap_qd, q_full + tb, bx * G::BOX,
                      w.sq.q0 + w.row0, w.h, w.sq.tb);
        ++tcn;
        for (int j = 0; j < w.n_kv; ++j, ++gj) {
          const int s = gj % C::NST;
          const uint32_t u = uint32_t(gj / C::NST);
          if (u > 0 && !mbar_wait(kv_empty + s, (u - 1) & 1, ctl, 131)) { ok = false; break; }
          mbar_arrive_expect_tx(kv_full + s, C::KV_TILE_BYTES);
          for (int bx = 0; bx < G::NBOX; ++bx)
            tma_load_4d(smem + kv_off + s * C::KV_TILE_BYTES + bx * BN * G::SW, tmap_kv, kv_full + s, bx * G::BOX,
                        w.sq.k0 + (w.kt0 + j) * BN, w.kvh, w.sq.tb);
        }
      }
      for (int i = (tcn > C::QB ? tcn - C::QB : 0); i < tcn; ++i)
        mbar_wait_drain(q_full + i % C::QB, uint32_t(i / C::QB) & 1, ctl, 132);
      for (int j = (gj > C::NST ? gj - C::NST : 0); j < gj; ++j)
        mbar_wait_drain(kv_full + j % C::NST, uint32_t(j / C::NST) & 1, ctl, 133);
    }
  } else if (warp == 1) {
    // =================== tcgen05 MMA issuer ===================
    if (lane == 0) {
      constexpr uint32_t IDESC_S = idesc_f16_f32(BM, BN, 0, 0, DT);
      constexpr uint32_t IDESC_DQ = idesc_f16_f32(BM, D, 0, 1, DT);
      auto k_tile = [&](int j) { return sbase + C::OFF_K + (j % C::NST) * C::KV_TILE_BYTES; };
      auto v_tile = [&](int j) { return sbase + C::OFF_V + (j % C::NST) * C::KV_TILE_BYTES; };
      auto wait_kv = [&](int j, int site) {
        const bool r = mbar_wait(kv_full + j % C::NST, uint32_t(j / C::NST) & 1, ctl, site);
        tc_fence_after();
        return r;
      };
      auto a_col = [](int ks) { return uint32_t((ks >> 2) * 64 + (ks & 3) * 8); };
      int gj = 0, tcn = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int t = snake_unit(cta, k, n_cta, n_tiles);
        if (t >= n_tiles) break;
        const int n_kv = tile_of<WIN>(shp, t).n_kv;
        if (n_kv == 0) continue;
        const int tb = tcn % C::QB;
        if (!mbar_wait(q_full + tb, uint32_t(tcn / C::QB) & 1, ctl, 140)) { ok = false; break; }
        tc_fence_after();
        const SDesc qd = desc_k_base<D>(sbase + C::OFF_Q + tb * C::Q_TILE_BYTES);
        const SDesc dd = desc_k_base<D>(sbase + C::OFF_DO + tb * C::Q_TILE_BYTES);
        // S buffer / barrier parities follow the CTA-wide key-tile count g
        auto issue_s = [&](int g) {
          const SDesc kd = desc_k_base<D>(k_tile(g));
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
            umma_ss(tmem + (g & 1) * 128, sdesc_at(qd, k_major_off<D, BM>(ks)), sdesc_at(kd, k_major_off<D, BN>(ks)),
                    IDESC_S, ks > 0);
          umma_commit(s_full + (g & 1));
        };
        auto issue_dp = [&](int g) {
          const SDesc vd = desc_k_base<D>(v_tile(g));
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
            umma_ss(tmem + C::DP_COL, sdesc_at(dd, k_major_off<D, BM>(ks)), sdesc_at(vd, k_major_off<D, BN>(ks)),
                    IDESC_S, ks > 0);
          umma_commit(dp_full);
        };
        if (!wait_kv(gj, 141)) { ok = false; break; }
        issue_s(gj);
        issue_dp(gj);
        if (n_kv > 1) {
          if (!wait_kv(gj + 1, 142)) { ok = false; break; }
          issue_s(gj + 1);
        }
        for (int j = 0; j < n_kv; ++j) {
          const int g = gj + j;
          if (!mbar_wait(ds_ready + (g & 1), uint32_t(g >> 1) & 1, ctl, 143)) { ok = false; break; }
          // dQ of the previous tile was read by the epilogue
          if (j == 0 && tcn > 0 && !mbar_wait(dq_empty, uint32_t(tcn - 1) & 1, ctl, 146)) { ok = false; break; }
          tc_fence_after();
          {
            const SDesc kd = desc_mn_base<D, BN>(k_tile(g));
            const uint32_t pa = tmem + (g & 1) * 128;
            umma_ts(tmem + C::DQ_COL, pa, sdesc_at(kd, 0), IDESC_DQ, j > 0 ? 1u : 0u);
#pragma unroll
            for (int ks = 1; ks < BN / 16; ++ks)
              umma_ts(tmem + C::DQ_COL, pa + a_col(ks), sdesc_at(kd, mn_major_off<D>(ks)), IDESC_DQ, 1u);
          }
          umma_commit(kv_empty + g % C::NST);
          if (j + 1 < n_kv) issue_dp(g + 1);  // its stage was waited for before S(g+1)
          if (j + 2 < n_kv) {
            if (!wait_kv(g + 2, 144)) { ok = false; break; }
            issue_s(g + 2);
          }
        }
        if (!ok) break;
        umma_commit(dq_full);
        umma_commit(q_empty + tb);
        gj += n_kv;
        ++tcn;
      }
      umma_commit(mma_done);
      mbar_wait_drain(mma_done, 0, ctl, 145);
    }
  } else if (warp >= 4) {
    // =================== dS warpgroups ===================
    const int w = (warp - 4) / 4;  // key-column half of every tile
    const int wq = warp & 3;
    const uint32_t lane_base = tmem_addr(tmem, uint32_t(wq * 32), 0);
    const uint64_t c2x2 = f2pack(shp.scale_log2, shp.scale_log2);
    // lse2 / Delta of this thread's row for the next tile are loaded one tile
    // ahead, so their latency hides behind the current tile.
    auto row_vals = [&](const Tile& wt, float& l, float& d) {
      const int r = wt.row0 + wq * 32 + lane;
      l = INFINITY;
      d = 0.f;
      if (r < wt.sq.nq && wt.n_kv > 0) {
        const long long i = row_stat_index(shp, wt.sq, wt.b, wt.h, r);
        const float x = lse[i];
        l = x == -INFINITY ? INFINITY : x;
        d = delta[i];
      }
    };
    int t_cur = snake_unit(cta, 0, n_cta, n_tiles);
    Tile wt = tile_of<WIN>(shp, t_cur < n_tiles ? t_cur : 0);
    float lse_n = INFINITY, delta_n = 0.f;
    if (t_cur < n_tiles) row_vals(wt, lse_n, delta_n);
    int gj = 0, tcn = 0;
    bool ok = true;
    for (int k = 0; ok && t_cur < n_tiles; ++k) {
      const Tile cur = wt;
      const float lse_r = lse_n, delta_r = delta_n;
      t_cur = snake_unit(cta, k + 1, n_cta, n_tiles);
      if (t_cur < n_tiles) {
        wt = tile_of<WIN>(shp, t_cur);
        row_vals(wt, lse_n, delta_n);
      }
      const int r = cur.row0 + wq * 32 + lane;
      int lim = cur.sq.nk - 1;
      long long lo = 0;  // first visible key under a sliding window
      if (shp.causal) {
        const long long c = (long long)r + shp.q_off - shp.k_off;
        lim = c < lim ? int(c) : lim;
        if (WIN) lo = c - shp.window + 1;
      }
      // dense boolean mask: this row's bit words (a row past the queries reads the last one)
      const uint32_t* mrow = nullptr;
      if constexpr (BITS) {
        const int rr = r < cur.sq.nq ? r : cur.sq.nq - 1;
        mrow = mk.bits + (long long)cur.b * mk.sb + (long long)cur.h * mk.sh + (long long)rr * mk.sn;
      }
      const uint64_t nlse2 = f2pack(-lse_r, -lse_r);
      const uint64_t ndelta2 = f2pack(-delta_r, -delta_r);
      // dropout: dS = P (Z r dP - Delta), Z = 1 where the position's byte is kept
      uint32_t drop_kbh = 0, nd_pk = 0;
      const int drop_b0 = 2 * (r & 1);
      uint64_t r2 = 0;
      if constexpr (DROP) {
        drop_kbh = drop_key_bh(dr, cur.b * shp.Hq + cur.h);
        nd_pk = pack2_f2<DT>(ndelta2);
        r2 = f2pack(dr.r, dr.r);
      }
      // mask words are loaded one key tile ahead
      uint2 mw_next;
      if constexpr (BITS) {
        if (cur.n_kv > 0) mw_next = __ldg(reinterpret_cast<const uint2*>(mrow + ((cur.kt0 * BN + 64 * w) >> 5)));
      }
      for (int j = 0; j < cur.n_kv; ++j) {
        const int g = gj + j;
        uint2 mw;
        if constexpr (BITS) {
          mw = mw_next;
          if (j + 1 < cur.n_kv)
            mw_next = __ldg(reinterpret_cast<const uint2*>(mrow + (((cur.kt0 + j + 1) * BN + 64 * w) >> 5)));
        }
        if (!mbar_wait_warp(s_full + (g & 1), uint32_t(g >> 1) & 1, ctl, 150 + w)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tS = lane_base + uint32_t((g & 1) * 128 + 64 * w);
        float sv[64];
        tmem_ld64(tS, sv);
        const int key0 = (cur.kt0 + j) * BN + 64 * w;  // key index of this half's column 0
        const int lim_j = lim - key0;                   // last visible column of this half
        if (lim_j < 63) {
#pragma unroll
          for (int c = 0; c < 64; ++c) sv[c] = c <= lim_j ? sv[c] : -INFINITY;
        }
        if (WIN && lo > key0) {
          const long long lo_j = lo - key0;
#pragma unroll
          for (int c = 0; c < 64; ++c) sv[c] = c >= lo_j ? sv[c] : -INFINITY;
        }
        if constexpr (BITS) {
          const uint32_t words[2] = {mw.x, mw.y};
          if ((words[0] & words[1]) != 0xffffffffu) apply_mask_bits<64>(sv, words);
        }
        // P in fp32, kept in place of the scores: dS = P (dP - Delta) is
        // formed in fp32 and rounded once, as the reference's
        // ds = p * (dp - Di) before .to(float16) (attention.py:343-347)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const uint64_t x = ffma2(f2pack(sv[2 * i], sv[2 * i + 1]), c2x2, nlse2);
          f2unpack((i & 7) < POLY_MASK ? exp2_poly2(x) : exp2_mufu2(x), sv[2 * i], sv[2 * i + 1]);
        }
        if (!mbar_wait_warp(dp_full, uint32_t(g) & 1, ctl, 152 + w)) { ok = false; break; }
        tc_fence_after();
        uint32_t pk_ds[32];
        if constexpr (DROP) {
          uint32_t pk_p[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) pk_p[i] = pack2<DT>(sv[2 * i], sv[2 * i + 1]);
          float dp[64];
          tmem_ld64(lane_base + uint32_t(C::DP_COL + 64 * w), dp);
          const uint32_t k2 = drop_key2(drop_kbh, r, key0);
          const uint32_t sel = drop_b0 ? keep_sel(2, 3) : keep_sel(0, 1);
          const uint32_t tt = (256u - dr.t) * 0x10001u;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            uint32_t w2[2];
            shared_words(drop_word(k2, r, key0 + 4 * j + 2 * (r & 1)), r & 1, w2[0], w2[1]);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int i = 2 * j + h;
              const uint32_t m = keep_mask2(w2[h], sel, tt);
              const uint32_t dk = pack2_f2<DT>(ffma2(f2pack(dp[2 * i], dp[2 * i + 1]), r2, ndelta2));
              pk_ds[i] = mul2<DT>(pk_p[i], (dk & m) | (nd_pk & ~m));
            }
          }
        } else {
#pragma unroll
          for (int hd = 0; hd < 2; ++hd) {
            float dp[32];
            tmem_ld32(lane_base + uint32_t(C::DP_COL + 64 * w + 32 * hd), dp);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int ii = 16 * hd + i;
              pk_ds[ii] = pack2_f2<DT>(fmul2(f2pack(sv[2 * ii], sv[2 * ii + 1]),
                                             fadd2(f2pack(dp[2 * i], dp[2 * i + 1]), ndelta2)));
            }
          }
        }
        tmem_st16(tS, *reinterpret_cast<uint32_t(*)[16]>(&pk_ds[0]));
        tmem_st16(tS + 16, *reinterpret_cast<uint32_t(*)[16]>(&pk_ds[16]));
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(ds_ready + (g & 1));
      }
      if (!ok) break;
      // ---- epilogue of the tile: warpgroup w stores dQ columns [w*D/2, (w+1)*D/2) ----
      if (cur.n_kv > 0) {
        if (!mbar_wait_warp(dq_full, uint32_t(tcn) & 1, ctl, 154 + w)) { ok = false; break; }
        tc_fence_after();
      }
      const float sc = shp.scale;
      constexpr int HALF = D / 2;
      float gv[HALF];
      if (cur.n_kv > 0) {
        if constexpr (HALF == 64) {
          tmem_ld64(lane_base + uint32_t(C::DQ_COL + w * HALF), *reinterpret_cast<float(*)[64]>(&gv[0]));
        } else if constexpr (HALF == 32) {
          tmem_ld32(lane_base + uint32_t(C::DQ_COL + w * HALF), *reinterpret_cast<float(*)[32]>(&gv[0]));
        } else {
          tmem_ld16(lane_base + uint32_t(C::DQ_COL + w * HALF), *reinterpret_cast<float(*)[16]>(&gv[0]));
        }
        tc_fence_before();
        mbar_arrive(dq_empty);
      } else {
#pragma unroll
        for (int i = 0; i < HALF; ++i) gv[i] = 0.f;
      }
      if (r < cur.sq.nq) {
        const long long off =
            (long long)cur.sq.tb * dq_sb + (long long)cur.h * dq_sh + (long long)(cur.sq.q0 + r) * dq_sn + w * HALF;
        if (accumulate_fp32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(dq_out) + off);
#pragma unroll
          for (int v4 = 0; v4 < HALF / 4; ++v4) {
            if (w * HALF + v4 * 4 >= shp.qk_cols) break;
            float4 x = dst[v4];
            x.x += gv[v4 * 4 + 0] * sc;
            x.y += gv[v4 * 4 + 1] * sc;
            x.z += gv[v4 * 4 + 2] * sc;
            x.w += gv[v4 * 4 + 3] * sc;
            dst[v4] = x;
          }
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(dq_out) + off);
#pragma unroll
          for (int v8 = 0; v8 < HALF / 8; ++v8) {
            if (w * HALF + v8 * 8 >= shp.qk_cols) break;
            uint4 pk;
            pk.x = pack2<DT>(gv[v8 * 8 + 0] * sc, gv[v8 * 8 + 1] * sc);
            pk.y = pack2<DT>(gv[v8 * 8 + 2] * sc, gv[v8 * 8 + 3] * sc);
            pk.z = pack2<DT>(gv[v8 * 8 + 4] * sc, gv[v8 * 8 + 5] * sc);
            pk.w = pack2<DT>(gv[v8 * 8 + 6] * sc, gv[v8 * 8 + 7] * sc);
            dst[v8] = pk;
          }
        }
      }
      if (cur.n_kv > 0) {
        gj += cur.n_kv;
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

template <int D, int DT, bool WIN, bool BITS = false, bool DROP = false>
int launch_bwd_dq_wide_t(const BwdArgs& a) {
  using C = bdqw::Cfg<D>;
  auto kern = fa_bwd_dq_wide_kernel<D, DT, WIN, BITS, DROP>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) != cudaSuccess)
    return FA_ERR_LAUNCH;
  const int n_qt = (a.shape.Nq + bdqw::BM - 1) / bdqw::BM;
  const int n_tiles = n_qt * a.shape.B * a.shape.Hq;
  const int sms = device_sm_count();
  const int n_cta = n_tiles < sms ? n_tiles : sms;
  kern<<<dim3(unsigned(n_cta)), bdqw::NUM_THREADS, C::SMEM_BYTES, a.stream>>>(
      a.tmap_q, a.tmap_do, a.tmap_k, a.tmap_v, a.shape, a.lse, a.delta, a.dq, a.dq_sb, a.dq_sh, a.dq_sn,
      a.accumulate_fp32, n_tiles, a.mask, a.drop);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

// Sliding-window, boolean and plain masks are separate instantiations.
template <int D, int DT>
int launch_bwd_dq_l(const BwdArgs& a) {
  if (a.drop.t) return launch_bwd_dq_wide_t<D, DT, false, false, true>(a);  // dense, no mask or window
  if (a.mask.bits) return launch_bwd_dq_wide_t<D, DT, false, true>(a);  // dense, no window
  return a.shape.window > 0 ? launch_bwd_dq_wide_t<D, DT, true>(a) : launch_bwd_dq_wide_t<D, DT, false>(a);
}

int launch_bwd_dq(const BwdArgs& a, int D) {
  switch (D) {
    case 32: return a.dtype == DT_BF16 ? launch_bwd_dq_l<32, DT_BF16>(a) : launch_bwd_dq_l<32, DT_F16>(a);
    case 64: return a.dtype == DT_BF16 ? launch_bwd_dq_l<64, DT_BF16>(a) : launch_bwd_dq_l<64, DT_F16>(a);
    case 128: return a.dtype == DT_BF16 ? launch_bwd_dq_l<128, DT_BF16>(a) : launch_bwd_dq_l<128, DT_F16>(a);
    default: return FA_ERR_UNSUPPORTED_HEAD_DIM;
  }
}

}  // namespace fa
