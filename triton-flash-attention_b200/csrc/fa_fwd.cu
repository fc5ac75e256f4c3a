// fa_fwd.cu -- FlashAttention-2 forward for B200 (sm_100a).
//
// Same result as the reference's _attn_fwd (triton_flash_attention/
// attention.py:90-234): O = softmax(scale * Q K^T [+ causal]) V and the base-2
// log-sum-exp lse2 = m + log2(l) per query row (attention.py:230).  The
// design is Blackwell-native rather than a translation:
//
//  * a work unit is 2 query tiles of 128 rows (256 rows) of one (batch,
//    head); the kernel is persistent: one CTA per SM walks its share of the
//    units back to back, so the next unit's Q load and first S MMAs overlap
//    the current unit's last key tiles and its epilogue (Q is
//    double-buffered where shared memory allows, D <= 64);
//  * warps 0 and 3 stream K and V tiles of 128 keys through a ring of
//    shared-memory stages with TMA (128- or 64-byte swizzle);
//  * warp 1 (one thread) issues tcgen05.mma: S_t = Q_t K^T into TMEM, then
//    O_t += P_t V with P_t read straight from TMEM (fp16);
//  * warps 4-7 and 8-11 are the softmax warpgroups of tile 0 and tile 1, one
//    thread per query row: they read S from TMEM, run the online softmax in
//    the base-2 domain (exp2 with scale * log2(e) folded in, as
//    attention.py:68-74), write P back to TMEM and rescale O in TMEM when the
//    running maximum grows by more than 2^8 (lazy rescaling);
//  * the softmax arithmetic is packed: a 3-input max tree and fma.rn.f32x2
//    for s * scale*log2(e) - m; the exponentials run on the MUFU unit
//    (ex2.approx, 16 per clock per SM).  A share of them can go to a
//    polynomial on the FMA pipe (POLY_MASK); measured, that does not pay
//    here;
//  * D <= 64 (TMEM to spare): P_t has its own TMEM buffer, so S_t of the
//    next key tile is issued as soon as the warpgroup has read S_t (not after
//    P_t V), and the warpgroup finds it ready when it finishes P_t.  The two
//    warpgroups take turns at their exponentials (tile 0, tile 1, tile 0,
//    ...), so that one's S reads, row maxima and P writes overlap the other's
//    exponentials instead of both contending for MUFU and then idling
//    together.  D = 128: P_t aliases S_t, and S_t(j+1) follows P_t(j) V.
// TMEM: S_0 cols [0,128), S_1 [128,256), O_0 [256,256+D), O_1 [256+D,256+2D),
// and for D <= 64 P_0 [256+2D, 320+2D), P_1 [320+2D, 384+2D).
#include "fa_common.cuh"
#include "fa_kernels.h"

namespace fa {

namespace fwd {

constexpr int BM = 128;  // query rows per tile
constexpr int BN = 128;  // keys per K/V tile
constexpr int QT = 2;    // query tiles per work unit
constexpr int NUM_THREADS = 384;
constexpr bool TURNS = true;  // separate-P layout: the softmax warpgroups take turns at their exponentials
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units: P may reach 2^8 before O is rescaled
#ifndef FA_FWD_POLY_MASK
#define FA_FWD_POLY_MASK 0
#endif
#ifndef FA_FWD_POLY_MASK_D32
#define FA_FWD_POLY_MASK_D32 2
#endif
constexpr int POLY_MASK = FA_FWD_POLY_MASK;          // pairs (i & 7) < POLY_MASK use the FMA-pipe exp2
constexpr int POLY_MASK_D32 = FA_FWD_POLY_MASK_D32;  // the same at D = 32 (half the MMA work per exponential; measured)
template <int D>
constexpr int poly_mask() { return D == 32 ? POLY_MASK_D32 : POLY_MASK; }
// Registers per thread: launched at 168 (384 threads); the control
// warpgroup (warps 0-3) drops to CTRL_REGS and the two softmax warpgroups
// rise to SOFT_REGS.  128 * CTRL_REGS + 256 * SOFT_REGS must not exceed
// 384 * 168 = 64512.
constexpr uint32_t LAUNCH_REGS = 168;
constexpr uint32_t CTRL_REGS = 64;
constexpr uint32_t SOFT_REGS = 216;
static_assert(128 * CTRL_REGS + 256 * SOFT_REGS <= NUM_THREADS * LAUNCH_REGS, "register split");

template <int D>
struct Cfg {
  using G = TileGeom<D>;
  static constexpr int NST = D == 128 ? 2 : 3;
  static constexpr int QB = D == 128 ? 1 : 2;  // Q buffers (units in flight)
  static constexpr int Q_TILE_BYTES = BM * D * 2;
  static constexpr int Q_UNIT_BYTES = QT * Q_TILE_BYTES;
  static constexpr int KV_TILE_BYTES = BN * D * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + QB * Q_UNIT_BYTES;
  static constexpr int OFF_V = OFF_K + NST * KV_TILE_BYTES;
  static constexpr int OW = D;  // O columns in TMEM
  static constexpr int OFF_BAR = OFF_V + NST * KV_TILE_BYTES;
  // barriers: q_full[QB], q_empty[QB], k_full[NST], k_empty[NST], v_full[NST], v_empty[NST],
  //           s_full[QT], p_ready[QT], o_full[QT], o_empty[QT], s_read[QT], pv_done[QT], turn[QT], mma_done
  static constexpr int NUM_BARS = 2 * QB + 4 * NST + 7 * QT + 1;
  static constexpr int OFF_CTL = OFF_BAR + NUM_BARS * 8;
  static constexpr int OFF_MISC = OFF_CTL + 16;
  // + alignment slack; at least 116 KB so that one CTA (and its 512 TMEM
  // columns) owns each SM
  static constexpr int SMEM_USED = OFF_MISC + 16 + 1024;
  static constexpr int SMEM_BYTES = SMEM_USED > 116 * 1024 ? SMEM_USED : 116 * 1024;
  static constexpr int S_COL0 = 0;
  static constexpr int O_COL0 = QT * BN;
  static constexpr int TMEM_COLS = 512;
  static_assert(O_COL0 + QT * OW <= TMEM_COLS, "TMEM budget");
  // D <= 64 leaves TMEM room for a P buffer per query tile (BN/2 columns of
  // packed fp16 pairs) beside S: S of the next key tile is then issued as
  // soon as the softmax warpgroup has read S, instead of after P V, so the
  // warpgroup finds its next S ready when it finishes P.  At D = 128, P
  // aliases S.
  static constexpr bool SEP_P = D <= 64;
  static constexpr int P_COL0 = O_COL0 + QT * OW;
  static_assert(!SEP_P || P_COL0 + QT * BN / 2 <= TMEM_COLS, "TMEM budget (separate P)");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

// A work unit: QT query tiles of one (batch, head); n_kv[t] key tiles each.
// Units are numbered late query blocks first (the heavy ones under a causal
// mask).  With GQA packing (shp.pack_g = G > 1) a unit is one (batch, K/V
// head) instead: its tiles hold the G query heads of the group x R = 128 / G
// query rows (tile row = g * R + r), h is the group's first query head, and
// row0 / rows count query rows per head.
// Key tiles: the unit streams key tiles kt0 .. kt0 + n_max - 1 (local index
// j = 0 .. n_max - 1); tile t is active for local j in [js[t], n_kv[t])
// (js = 0 and kt0 = 0 unless a sliding window hides leading keys).
// With SPLIT, unit u is key range u / (units without the split) of unit
// u % (that count), and its key tiles are cut to that range.
struct Unit {
  int b, h, kvh, row0, rows, kt0, js[QT], n_kv[QT], n_max;
  int split;
  Seq sq;
};
template <bool PACK, bool WIN, bool SPLIT = false>
__device__ __forceinline__ Unit unit_of(const AttnShape& shp, int u, const SplitArgs& sp) {
  const int G = PACK ? shp.pack_g : 1;
  const int rows = BM / G;  // query rows per head in a tile
  const int BH = shp.B * (G > 1 ? shp.Hkv : shp.Hq);
  const int n_qblk = (shp.Nq + QT * rows - 1) / (QT * rows);
  Unit w;
  w.split = 0;
  if (SPLIT) {
    w.split = u / (BH * n_qblk);
    u -= w.split * (BH * n_qblk);
  }
  const int bh = u % BH;
  if (PACK) {
    w.b = bh / shp.Hkv;
    w.kvh = bh % shp.Hkv;
    w.h = w.kvh * G;
  } else {
    w.b = bh / shp.Hq;
    w.h = bh % shp.Hq;
    w.kvh = w.h / (shp.Hq / shp.Hkv);
  }
  w.rows = rows;
  w.row0 = (n_qblk - 1 - u / BH) * QT * rows;
  w.sq = seq_of(shp, w.b);
  int first[QT], end[QT];
  w.kt0 = 1 << 30;
#pragma unroll
  for (int t = 0; t < QT; ++t) {
    end[t] = kv_tiles_for_rows(shp, w.sq, w.row0 + t * rows, rows, BN);
    first[t] = WIN ? kv_first_tile(shp, w.sq, w.row0 + t * rows, BN) : 0;
    if (SPLIT) {
      const int lo = w.split * sp.tiles;
      first[t] = first[t] > lo ? first[t] : lo;
      end[t] = end[t] < lo + sp.tiles ? end[t] : lo + sp.tiles;
    }
    if (first[t] >= end[t]) first[t] = end[t] = 0;  // no visible key
    else w.kt0 = first[t] < w.kt0 ? first[t] : w.kt0;
  }
  if (w.kt0 == (1 << 30)) w.kt0 = 0;
  w.n_max = 0;
#pragma unroll
  for (int t = 0; t < QT; ++t) {
    const bool active = end[t] > first[t];
    w.js[t] = active ? first[t] - w.kt0 : 0;
    w.n_kv[t] = active ? end[t] - w.kt0 : 0;
    w.n_max = w.n_kv[t] > w.n_max ? w.n_kv[t] : w.n_max;
  }
  return w;
}

}  // namespace fwd

template <int D, int DT, bool PACK, bool WIN, bool BITS, bool DROP, bool SPLIT>
__global__ void __launch_bounds__(fwd::NUM_THREADS, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                  const __grid_constant__ CUtensorMap tmap_v, const AttnShape shp, uint16_t* __restrict__ o_ptr,
                  const long long o_sb, const long long o_sh, const long long o_sn, float* __restrict__ lse_ptr,
                  const int n_units, const MaskBits mk, const DropArgs dr, const SplitArgs sp) {
  using namespace fwd;
  using C = Cfg<D>;
  using G = TileGeom<D>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled TMA destinations.
  const uint32_t raw_saddr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_saddr + 1023u) & ~1023u) - raw_saddr);
  const uint32_t sbase = smem_u32(smem);

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + C::QB;
  uint64_t* k_full = q_empty + C::QB;
  uint64_t* k_empty = k_full + C::NST;
  uint64_t* v_full = k_empty + C::NST;
  uint64_t* v_empty = v_full + C::NST;
  // per query tile t: s_full / p_ready complete once per key tile of t,
  // o_full / o_empty once per unit in which t sees a key
  uint64_t* s_full = v_empty + C::NST;
  uint64_t* p_ready = s_full + QT;
  uint64_t* o_full = p_ready + QT;
  uint64_t* o_empty = o_full + QT;
  // per query tile t (separate-P layout): s_read completes once the
  // warpgroup has read S_t into registers, pv_done once P_t V has run
  uint64_t* s_read = o_empty + QT;
  uint64_t* pv_done = s_read + QT;
  // turn[t]: the other softmax warpgroup finished its exponentials and
  // hands the MUFU unit to tile t's (one phase per hand-off)
  uint64_t* turn = pv_done + QT;
  uint64_t* mma_done = turn + QT;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  CtaCtl* ctl_w = reinterpret_cast<CtaCtl*>(smem + C::OFF_CTL);
  volatile CtaCtl* ctl = ctl_w;

  const int warp = int(warp_id());
  const int lane = int(lane_id());
  const int cta = int(blockIdx.x);
  const int n_cta = int(gridDim.x);

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::QB; ++i) {
      mbar_init(q_full + i, 1);
      mbar_init(q_empty + i, 1);
    }
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(k_empty + s, 1);
      mbar_init(v_full + s, 1);
      mbar_init(v_empty + s, 1);
    }
    for (int t = 0; t < QT; ++t) {
      mbar_init(s_full + t, 1);
      mbar_init(p_ready + t, 128);
      mbar_init(o_full + t, 1);
      mbar_init(o_empty + t, 128);
      mbar_init(s_read + t, 128);
      mbar_init(pv_done + t, 1);
    }
    for (int t = 0; t < QT; ++t) mbar_init(turn + t, 128);
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
      // =================== TMA producers ===================
      // Warp 0 loads Q and the K tiles, warp 3 the V tiles: one thread's TMA
      // loads are processed one after another (~0.5 us per 16 KB box measured),
      // so K and V come from two threads to double the stream rate.
      const bool is_k = warp == 0;
      if (lane == 0) {
        const CUtensorMap* tmap_kv = is_k ? &tmap_k : &tmap_v;
        uint64_t* kv_full = is_k ? k_full : v_full;
        uint64_t* kv_empty = is_k ? k_empty : v_empty;
        const int kv_off = is_k ? C::OFF_K : C::OFF_V;
        tma_prefetch_desc(tmap_kv);
        if (is_k) tma_prefetch_desc(&tmap_q);
        int gj = 0, uc = 0;  // key tiles and non-empty units issued
        bool ok = true;
        for (int k = 0; ok; ++k) {
          const int ui = snake_unit(cta, k, n_cta, n_units);
          if (ui >= n_units) break;
          const Unit w = unit_of<PACK, WIN, SPLIT>(shp, ui, sp);
          if (w.n_max == 0) continue;
          if (is_k) {
            const int qb = uc % C::QB;
            if (uc >= C::QB && !mbar_wait(q_empty + qb, uint32_t(uc / C::QB - 1) & 1, ctl, 6)) break;
            int q_bytes = 0;
            for (int t = 0; t < QT; ++t) q_bytes += w.n_kv[t] > 0 ? C::Q_TILE_BYTES : 0;
            mbar_arrive_expect_tx(q_full + qb, q_bytes);
            for (int t = 0; t < QT; ++t) {
              if (w.n_kv[t] == 0) continue;
              for (int bx = 0; bx < G::NBOX; ++bx)
                tma_load_4d(smem + C::OFF_Q + qb * C::Q_UNIT_BYTES + t * C::Q_TILE_BYTES + bx * BM * G::SW, &tmap_q,
                            q_full + qb, bx * G::BOX, w.sq.q0 + w.row0 + t * w.rows, w.h, w.sq.tb);
            }
          }
          ++uc;
          for (int j = 0; j < w.n_max; ++j, ++gj) {
            const int s = gj % C::NST;
            const uint32_t u = uint32_t(gj / C::NST);
            if (u > 0 && !mbar_wait(kv_empty + s, (u - 1) & 1, ctl, is_k ? 1 : 2)) { ok = false; break; }
            mbar_arrive_expect_tx(kv_full + s, C::KV_TILE_BYTES);
            if (shp.block_table) {
              // paged K/V: the tile's 128 keys in pieces of min(page, 128)
              // rows, one load per page; pieces past the batch's last page
              // repeat it (finite data; their keys are masked)
              const int P = shp.page_size;
              const int PR = P < BN ? P : BN;
              const int last_page = (w.sq.nk - 1) / P;
              const int* bt = shp.block_table + (long long)w.b * shp.bt_stride;
              for (int i = 0; i < BN / PR; ++i) {
                const int kr = (w.kt0 + j) * BN + i * PR;
                const int pidx = kr / P < last_page ? kr / P : last_page;
                const int row = __ldg(bt + pidx) * P + kr % P;
                for (int bx = 0; bx < G::NBOX; ++bx)
                  tma_load_4d(smem + kv_off + s * C::KV_TILE_BYTES + bx * BN * G::SW + i * PR * G::SW, tmap_kv,
                              kv_full + s, bx * G::BOX, row, w.kvh, 0);
              }
            } else {
              for (int bx = 0; bx < G::NBOX; ++bx)
                tma_load_4d(smem + kv_off + s * C::KV_TILE_BYTES + bx * BN * G::SW, tmap_kv, kv_full + s,
                            bx * G::BOX, w.sq.k0 + (w.kt0 + j) * BN, w.kvh, w.sq.tb);
            }
          }
        }
        // Drain: every load this thread issued must land before the CTA exits.
        // On the normal path these phases have completed already.
        if (is_k)
          for (int i = (uc > C::QB ? uc - C::QB : 0); i < uc; ++i)
            mbar_wait_drain(q_full + i % C::QB, uint32_t(i / C::QB) & 1, ctl, 3);
        for (int j = (gj > C::NST ? gj - C::NST : 0); j < gj; ++j)
          mbar_wait_drain(kv_full + j % C::NST, uint32_t(j / C::NST) & 1, ctl, is_k ? 4 : 5);
      }
    } else if (warp == 1) {
      // =================== tcgen05 MMA issuer ===================
      if (lane == 0) {
        constexpr uint32_t IDESC_S = idesc_f16_f32(BM, BN, 0, 0, DT);
        constexpr uint32_t IDESC_PV = idesc_f16_f32(BM, C::OW, 0, 1, DT);
        const uint32_t k_s = sbase + C::OFF_K;
        const uint32_t v_s = sbase + C::OFF_V;
        int gj = 0, uc = 0;
        int cnt[QT] = {0, 0};  // key tiles of query tile t so far (s_full / p_ready phases)
        int oc[QT] = {0, 0};   // units in which tile t saw a key (o_full / o_empty phases)
        bool ok = true;
        for (int k = 0; ok; ++k) {
          const int ui = snake_unit(cta, k, n_cta, n_units);
          if (ui >= n_units) break;
          const Unit w = unit_of<PACK, WIN, SPLIT>(shp, ui, sp);
          if (w.n_max == 0) continue;
          const int qb = uc % C::QB;
          if (!mbar_wait(q_full + qb, uint32_t(uc / C::QB) & 1, ctl, 10)) { ok = false; break; }
          // descriptor bases (the issue loops below only add constants)
          SDesc qd[QT];
  #pragma unroll
          for (int t = 0; t < QT; ++t) qd[t] = desc_k_base<D>(sbase + C::OFF_Q + qb * C::Q_UNIT_BYTES + t * C::Q_TILE_BYTES);
          auto issue_s = [&](int t, int g) {
            const SDesc kd = desc_k_base<D>(k_s + (g % C::NST) * C::KV_TILE_BYTES);
            const uint32_t dst = tmem + C::S_COL0 + t * BN;
  #pragma unroll
            for (int ks = 0; ks < D / 16; ++ks)
              umma_ss(dst, sdesc_at(qd[t], k_major_off<D, BM>(ks)), sdesc_at(kd, k_major_off<D, BN>(ks)), IDESC_S,
                      ks > 0);
            umma_commit(s_full + t);
          };
          auto issue_pv = [&](int t, int g, bool acc) {
            // the D columns of V span NBOX boxes BN*SW bytes apart (LBO)
            const SDesc vd = desc_mn_base<D, BN>(v_s + (g % C::NST) * C::KV_TILE_BYTES);
            const uint32_t dst = tmem + C::O_COL0 + t * C::OW;
            const uint32_t pa = C::SEP_P ? tmem + C::P_COL0 + t * (BN / 2) : tmem + C::S_COL0 + t * BN;
            umma_ts(dst, pa, sdesc_at(vd, 0), IDESC_PV, acc ? 1u : 0u);
  #pragma unroll
            for (int ks = 1; ks < BN / 16; ++ks)
              umma_ts(dst, pa + ks * 8, sdesc_at(vd, mn_major_off<D>(ks)), IDESC_PV, 1u);
          };
          if (!mbar_wait(k_full + gj % C::NST, uint32_t(gj / C::NST) & 1, ctl, 11)) { ok = false; break; }
          tc_fence_after();
          for (int t = 0; t < QT; ++t)
            if (w.n_kv[t] > 0 && w.js[t] == 0) issue_s(t, gj);
          umma_commit(k_empty + gj % C::NST);
          if constexpr (C::SEP_P) {
            // S_t(j+1) once the warpgroup read S_t(j); P_t(j) V once it wrote P_t(j)
            for (int j = 0; j < w.n_max && ok; ++j) {
              const int g = gj + j;
              const int s = g % C::NST;
              const bool more = j + 1 < w.n_max;
              if (more) {
                if (!mbar_wait(k_full + (g + 1) % C::NST, uint32_t((g + 1) / C::NST) & 1, ctl, 13)) { ok = false; break; }
                for (int t = 0; t < QT && ok; ++t) {
                  if (j + 1 >= w.n_kv[t] || j + 1 < w.js[t]) continue;
                  // a tile's first S in the unit finds its buffer free; later
                  // ones wait until the warpgroup read the previous S
                  if (j + 1 > w.js[t] && !mbar_wait(s_read + t, uint32_t(cnt[t]) & 1, ctl, 17)) { ok = false; break; }
                  tc_fence_after();
                  issue_s(t, g + 1);
                }
                if (!ok) break;
                umma_commit(k_empty + (g + 1) % C::NST);
              }
              if (!mbar_wait(v_full + s, uint32_t(g / C::NST) & 1, ctl, 12)) { ok = false; break; }
              for (int t = 0; t < QT && ok; ++t) {
                if (j >= w.n_kv[t] || j < w.js[t]) continue;
                if (!mbar_wait(p_ready + t, uint32_t(cnt[t]) & 1, ctl, 14)) { ok = false; break; }
                if (j == w.js[t] && oc[t] > 0 && !mbar_wait(o_empty + t, uint32_t(oc[t] - 1) & 1, ctl, 16)) { ok = false; break; }
                tc_fence_after();
                issue_pv(t, g, j > w.js[t]);
                umma_commit(pv_done + t);
                ++cnt[t];
              }
              if (!ok) break;
              umma_commit(v_empty + s);
            }
          } else
          for (int j = 0; j < w.n_max && ok; ++j) {
            const int g = gj + j;
            const int s = g % C::NST;
            if (!mbar_wait(v_full + s, uint32_t(g / C::NST) & 1, ctl, 12)) { ok = false; break; }
            const bool more = j + 1 < w.n_max;
            if (more && !mbar_wait(k_full + (g + 1) % C::NST, uint32_t((g + 1) / C::NST) & 1, ctl, 13)) {
              ok = false;
              break;
            }
            tc_fence_after();
            for (int t = 0; t < QT && ok; ++t) {
              if (j + 1 == w.js[t] && j + 1 < w.n_kv[t]) issue_s(t, g + 1);  // the tile's first S
              if (j >= w.n_kv[t] || j < w.js[t]) continue;
              if (!mbar_wait(p_ready + t, uint32_t(cnt[t]) & 1, ctl, 14)) { ok = false; break; }
              // O_t of the previous unit was read by its epilogue
              if (j == w.js[t] && oc[t] > 0 && !mbar_wait(o_empty + t, uint32_t(oc[t] - 1) & 1, ctl, 16)) { ok = false; break; }
              tc_fence_after();
              issue_pv(t, g, j > w.js[t]);
              ++cnt[t];
              if (j + 1 < w.n_kv[t]) issue_s(t, g + 1);
            }
            if (!ok) break;
            umma_commit(v_empty + s);
            if (more) umma_commit(k_empty + (g + 1) % C::NST);
          }
          if (!ok) break;
          for (int t = 0; t < QT; ++t)
            if (w.n_kv[t] > 0) {
              umma_commit(o_full + t);
              ++oc[t];
            }
          umma_commit(q_empty + qb);
          gj += w.n_max;
          ++uc;
        }
        // Drain every MMA this thread issued before the CTA tears down TMEM.
        umma_commit(mma_done);
        mbar_wait_drain(mma_done, 0, ctl, 15);
      }
    }
  } else {
    regs_claim<SOFT_REGS>();
    // =================== softmax warpgroups ===================
    const int t = (warp - 4) / 4;       // query tile of this warpgroup
    const int wq = warp & 3;            // TMEM lane quadrant this warp may access
    const int row_local = wq * 32 + lane;
    const uint32_t tS = tmem_addr(tmem, uint32_t(wq * 32), uint32_t(C::S_COL0 + t * BN));
    const uint32_t tO = tmem_addr(tmem, uint32_t(wq * 32), uint32_t(C::O_COL0 + t * C::OW));
    const uint32_t tP = tmem_addr(tmem, uint32_t(wq * 32), uint32_t(C::SEP_P ? C::P_COL0 + t * (BN / 2) : 0));
    const float c2 = shp.scale_log2;
    const uint64_t c2x2 = f2pack(c2, c2);
    int cnt = 0, oc = 0;  // phases of s_full / o_full of this tile
    // Turns: the exponential phases of the two warpgroups strictly
    // alternate, tile 0 first, (0, j), (1, j) for each key tile j of each
    // unit; a warpgroup with fewer key tiles in a unit takes empty turns.
    // While one warpgroup has the MUFU unit, the other reads its next S,
    // finds the row maxima and writes P, which keeps the MUFU unit busy
    // instead of both warpgroups contending for it and then idling together.
    int pc = 0;  // turns taken by this warpgroup
    auto take_turn = [&]() -> bool {
      if (t == 0 && pc == 0) return true;
      return mbar_wait_warp(turn + t, uint32_t(t == 0 ? pc - 1 : pc) & 1, ctl, 26 + t);
    };
    auto pass_turn = [&]() {
      mbar_arrive(turn + (1 - t));
      ++pc;
    };
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int ui = snake_unit(cta, k, n_cta, n_units);
      if (ui >= n_units) break;
      const Unit w = unit_of<PACK, WIN, SPLIT>(shp, ui, sp);
      // query row (within the batch) and head of this thread's tile row
      const int r = w.row0 + t * w.rows + (PACK ? row_local % w.rows : row_local);
      const int hq = w.h + (PACK ? row_local / w.rows : 0);
      const int nt = w.n_kv[t];  // this tile's steps are local key tiles js .. nt - 1
      const int js = w.js[t];
      // last visible key column of this row (key index in the batch), and
      // with a sliding window the first one
      int lim = w.sq.nk - 1;
      long long lo = 0;
      if (shp.causal) {
        const long long c = (long long)r + shp.q_off - shp.k_off + w.sq.diag;
        lim = c < lim ? int(c) : lim;  // may be negative: no visible key
        if (WIN) lo = c - shp.window + 1;
      }
      // dense boolean mask: this row's bit words (a row past the queries reads the last one)
      const uint32_t* mrow = nullptr;
      if constexpr (BITS) {
        const int rr = r < w.sq.nq ? r : w.sq.nq - 1;
        mrow = mk.bits + (long long)w.b * mk.sb + (long long)hq * mk.sh + (long long)rr * mk.sn;
      }
      if constexpr (C::SEP_P && TURNS) {
        // empty turns for the leading key tiles the other query tile has and this one lacks
        for (int j = 0; j < js && ok; ++j) {
          if (!take_turn()) { ok = false; break; }
          pass_turn();
        }
        if (!ok) break;
      }
      // dropout: this row's random-byte positions within a block word
      uint32_t drop_kbh = 0;
      const int drop_b0 = 2 * (r & 1);
      if constexpr (DROP) drop_kbh = drop_key_bh(dr, w.b * shp.Hq + hq);
      float m = -INFINITY;  // running exponent base (scaled log2 units)
      float l = 0.f;        // running row sum of exp2(s * c2 - m)
      // mask words are loaded one key tile ahead, so the load's latency hides behind a tile
      uint4 mw_next;
      if constexpr (BITS) {
        if (js < nt) mw_next = __ldg(reinterpret_cast<const uint4*>(mrow + (w.kt0 + js) * (BN / 32)));
      }
      for (int j = js; j < nt; ++j) {
        uint4 mw;
        if constexpr (BITS) {
          mw = mw_next;
          if (j + 1 < nt) mw_next = __ldg(reinterpret_cast<const uint4*>(mrow + (w.kt0 + j + 1) * (BN / 32)));
        }
        if (!mbar_wait_warp(s_full + t, uint32_t(cnt) & 1, ctl, 20 + t)) { ok = false; break; }
        tc_fence_after();
        float s[BN];
        tmem_ld64(tS, *reinterpret_cast<float(*)[64]>(&s[0]));
        tmem_ld64(tS + 64, *reinterpret_cast<float(*)[64]>(&s[64]));
        if constexpr (C::SEP_P) {
          // S_t is in registers: the MMA may overwrite it with the next key tile's
          tc_fence_before();
          mbar_arrive(s_read + t);
        }
        const int key0 = (w.kt0 + j) * BN;  // key index of this tile's column 0
        const int lim_j = lim - key0;      // last visible column in this tile
        if (lim_j < BN - 1) {
#pragma unroll
          for (int c = 0; c < BN; ++c) s[c] = c <= lim_j ? s[c] : -INFINITY;
        }
        if (WIN && lo > key0) {  // sliding window: columns before lo are hidden
          const long long lo_j = lo - key0;
#pragma unroll
          for (int c = 0; c < BN; ++c) s[c] = c >= lo_j ? s[c] : -INFINITY;
        }
        if constexpr (BITS) {
          const uint32_t words[4] = {mw.x, mw.y, mw.z, mw.w};
          // a tile row with every key visible needs no select
          if ((words[0] & words[1] & words[2] & words[3]) != 0xffffffffu) apply_mask_bits<BN>(s, words);
        }
        // row max: 8 independent 3-input max chains, then a short tree
        float a8[8];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          float acc = fmax3(s[kk * 16], s[kk * 16 + 1], s[kk * 16 + 2]);
#pragma unroll
          for (int i = 3; i < 15; i += 2) acc = fmax3(acc, s[kk * 16 + i], s[kk * 16 + i + 1]);
          a8[kk] = fmaxf(acc, s[kk * 16 + 15]);
        }
        const float mx = fmax3(fmax3(a8[0], a8[1], a8[2]), fmax3(a8[3], a8[4], a8[5]), fmaxf(a8[6], a8[7]));
        const float m_tile = mx * c2;
        bool rescale = false;
        float m_new = m;
        if (m_tile > m + RESCALE_THRESHOLD) {  // false while m_tile == -inf
          m_new = m_tile;
          rescale = true;
        }
        const float alpha = rescale ? ex2(m - m_new) : 1.f;  // ex2(-inf) = 0 on the first tile
        const float base = m_new == -INFINITY ? 0.f : m_new;
        uint64_t nb2 = f2pack(-base, -base);
        if constexpr (C::SEP_P && TURNS) {
          if (!take_turn()) { ok = false; break; }
          asm volatile("" : "+l"(nb2));  // the exponentials below depend on the turn
        }
        uint64_t sum2[4] = {0, 0, 0, 0};
        uint32_t pk[C::SEP_P ? BN / 2 : 1];  // P_t, packed, until the previous P_t V has run
        uint32_t drop_k2 = 0;
        if constexpr (DROP) drop_k2 = drop_key2(drop_kbh, r, key0);
#pragma unroll
        for (int cc = 0; cc < BN / 32; ++cc) {
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int c0 = cc * 32 + 2 * i;
            const uint64_t x = ffma2(f2pack(s[c0], s[c0 + 1]), c2x2, nb2);
            // POLY_MASK of every 8 pairs on the FMA pipe, the rest on MUFU
            const uint64_t e = (i & 7) < poly_mask<D>() ? exp2_poly2(x) : exp2_mufu2(x);
            packed[i] = pack2_f2<DT>(e);
            sum2[i & 3] = fadd2(sum2[i & 3], e);  // the row sum counts dropped values too
          }
          if constexpr (DROP) {
            const uint32_t sel = (r & 1) ? keep_sel(2, 3) : keep_sel(0, 1);
            const uint32_t tt = (256u - dr.t) * 0x10001u;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              uint32_t we, wo;
              shared_words(drop_word(drop_k2, r, key0 + cc * 32 + 4 * j + 2 * (r & 1)), r & 1, we, wo);
              packed[2 * j] &= keep_mask2(we, sel, tt);
              packed[2 * j + 1] &= keep_mask2(wo, sel, tt);
            }
          }
          if constexpr (C::SEP_P) {
#pragma unroll
            for (int i = 0; i < 16; ++i) pk[cc * 16 + i] = packed[i];
          } else {
            tmem_st16(tS + cc * 16, packed);
          }
        }
        if constexpr (C::SEP_P && TURNS) {
          // the turn ends once every exponential of this key tile is summed
          const uint64_t q01 = fadd2(fadd2(sum2[0], sum2[1]), fadd2(sum2[2], sum2[3]));
          asm volatile("" ::"l"(q01));
          pass_turn();
        }
        if constexpr (C::SEP_P) {
          // P_t(j-1) V has read the P buffer and finished accumulating O_t
          if (j > js && !mbar_wait_warp(pv_done + t, uint32_t(cnt - 1) & 1, ctl, 24 + t)) { ok = false; break; }
          tc_fence_after();
        }
        {
          float s0, s1, s2, s3, s4, s5, s6, s7;
          f2unpack(sum2[0], s0, s1);
          f2unpack(sum2[1], s2, s3);
          f2unpack(sum2[2], s4, s5);
          f2unpack(sum2[3], s6, s7);
          l = l * alpha + (((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7)));
        }
        m = m_new;
        if constexpr (C::SEP_P) {
#pragma unroll
          for (int cc = 0; cc < BN / 32; ++cc) tmem_st16(tP + cc * 16, *reinterpret_cast<uint32_t(*)[16]>(&pk[cc * 16]));
        }
        if (j > js && __any_sync(0xffffffffu, rescale)) {
          // O *= alpha
#pragma unroll 1
          for (int cc = 0; cc < C::OW / 16; ++cc) {
            float o[16];
            tmem_ld16(tO + cc * 16, o);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] *= alpha;
            uint32_t u[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) u[i] = __float_as_uint(o[i]);
            tmem_st16(tO + cc * 16, u);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(p_ready + t);
        ++cnt;
      }
      if (!ok) break;
      if constexpr (C::SEP_P && TURNS) {
        // empty turns for the key tiles the other query tile has and this one lacks
        for (int j = nt; j < w.n_max; ++j) {
          if (!take_turn()) { ok = false; break; }
          pass_turn();
        }
        if (!ok) break;
      }
      // ---- epilogue: O / l -> fp16, lse2 = m + log2(l) ----
      if (nt > 0) {
        if (!mbar_wait_warp(o_full + t, uint32_t(oc) & 1, ctl, 22 + t)) { ok = false; break; }
        tc_fence_after();
      }
      const bool row_ok = r < w.sq.nq;
      const float inv_l = (l > 0.f ? 1.f / l : 0.f) * (DROP ? dr.r : 1.f);
      uint16_t* orow = o_ptr + (long long)w.sq.tb * o_sb + (long long)hq * o_sh + (long long)(w.sq.q0 + r) * o_sn +
                       (SPLIT ? w.split * sp.o_stride : 0);
#pragma unroll 1
      for (int cc = 0; cc < D / 32; ++cc) {
        float o[32];
        if (nt > 0) {
          tmem_ld32(tO + cc * 32, o);
          if (cc == D / 32 - 1) {
            // O_t is read: the next unit's first PV may overwrite it
            tc_fence_before();
            mbar_arrive(o_empty + t);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (row_ok && cc * 32 < shp.v_cols) {
#pragma unroll
          for (int v8 = 0; v8 < 4; ++v8) {
            uint4 pk;
            pk.x = pack2<DT>(o[v8 * 8 + 0] * inv_l, o[v8 * 8 + 1] * inv_l);
            pk.y = pack2<DT>(o[v8 * 8 + 2] * inv_l, o[v8 * 8 + 3] * inv_l);
            pk.z = pack2<DT>(o[v8 * 8 + 4] * inv_l, o[v8 * 8 + 5] * inv_l);
            pk.w = pack2<DT>(o[v8 * 8 + 6] * inv_l, o[v8 * 8 + 7] * inv_l);
            *reinterpret_cast<uint4*>(orow + cc * 32 + v8 * 8) = pk;
          }
        }
      }
      if (nt > 0) ++oc;
      if (row_ok) {
        lse_ptr[row_stat_index(shp, w.sq, w.b, hq, r) + (SPLIT ? w.split * sp.lse_stride : 0)] =
            l > 0.f ? m + lg2(l) : -INFINITY;
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

template <int D, int DT, bool PACK, bool WIN, bool BITS = false, bool DROP = false, bool SPLIT = false>
int launch_fwd_t(const FwdArgs& a) {
  using C = fwd::Cfg<D>;
  const int smem = C::SMEM_BYTES;
  auto kern = fa_fwd_kernel<D, DT, PACK, WIN, BITS, DROP, SPLIT>;
  // The register split inside the kernel assumes the launch count; a build
  // that allocated a different number must not run (an increase that does
  // not fit would wait forever).
  static int regs_ok = -1;
  if (regs_ok < 0) {
    cudaFuncAttributes fa_attr;
    regs_ok = cudaFuncGetAttributes(&fa_attr, kern) == cudaSuccess && fa_attr.numRegs == int(fwd::LAUNCH_REGS) ? 1 : 0;
  }
  if (!regs_ok) return FA_ERR_LAUNCH;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return FA_ERR_LAUNCH;
  const int G = a.shape.pack_g > 1 ? a.shape.pack_g : 1;
  const int rows = fwd::QT * (fwd::BM / G);
  const int n_qblk = (a.shape.Nq + rows - 1) / rows;
  const int n_units = n_qblk * a.shape.B * (G > 1 ? a.shape.Hkv : a.shape.Hq) * (SPLIT ? a.split.n : 1);
  const int sms = device_sm_count();
  const int n_cta = n_units < sms ? n_units : sms;
  kern<<<dim3(unsigned(n_cta)), fwd::NUM_THREADS, smem, a.stream>>>(a.tmap_q, a.tmap_k, a.tmap_v, a.shape, static_cast<uint16_t*>(a.o),
                                                                    a.o_sb, a.o_sh, a.o_sn, a.lse, n_units, a.mask, a.drop,
                                                                    a.split);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

// GQA-packed and plain query tiles, and sliding-window, boolean and plain
// masks, are separate instantiations.
template <int D, int DT>
int launch_fwd_l(const FwdArgs& a) {
  // split-KV: GQA-packed, no mask, window or dropout (checked by the caller)
  if (a.split.n > 1) return launch_fwd_t<D, DT, true, false, false, false, true>(a);
  if (a.drop.t) return launch_fwd_t<D, DT, false, false, false, true>(a);  // dense, unpacked, no mask or window
  if (a.mask.bits) return launch_fwd_t<D, DT, false, false, true>(a);  // dense, unpacked, no window
  if (a.shape.window > 0)
    return a.shape.pack_g > 1 ? launch_fwd_t<D, DT, true, true>(a) : launch_fwd_t<D, DT, false, true>(a);
  return a.shape.pack_g > 1 ? launch_fwd_t<D, DT, true, false>(a) : launch_fwd_t<D, DT, false, false>(a);
}

int launch_fwd(const FwdArgs& a, int D) {
  switch (D) {
    case 32: return a.dtype == DT_BF16 ? launch_fwd_l<32, DT_BF16>(a) : launch_fwd_l<32, DT_F16>(a);
    case 64: return a.dtype == DT_BF16 ? launch_fwd_l<64, DT_BF16>(a) : launch_fwd_l<64, DT_F16>(a);
    case 128: return a.dtype == DT_BF16 ? launch_fwd_l<128, DT_BF16>(a) : launch_fwd_l<128, DT_F16>(a);
    default: return FA_ERR_UNSUPPORTED_HEAD_DIM;
  }
}

}  // namespace fa
