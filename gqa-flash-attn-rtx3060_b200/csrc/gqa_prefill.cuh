// tcgen05 / TMEM / TMA GQA forward for many packed query rows (prefill and
// chunked prefill).
//
// One CTA owns two 128-row query tiles of one (batch, kv_head). A tile packs
// the group's `group` query heads x `bm = 128 / group` consecutive positions
// into the 128 rows of one UMMA (row r -> head kv*group + r / bm, position
// p + r % bm), the group packing of gqa_kernels/gqa_fwd.py:57-65, done here by
// one 4-D TMA box {64, bm, group, 1}. K and V tiles of 128 keys stream through
// a ring of shared-memory slots filled by a TMA producer warp.
//
// Per key tile j and query tile i (i = 0, 1):
//   MMA warp (one thread):  S_i = Q_i K_j^T          (SS UMMA, f32 into TMEM)
//   softmax warpgroup i:    P_i = exp2(S_i*scale - m) (bf16/f16 written back into TMEM over S_i)
//   MMA warp:               O_i += P_i V_j            (TS UMMA: A = P from TMEM, B = V from smem)
// The two tiles ping-pong so one warpgroup's exp2 work overlaps the other
// tile's MMAs. The running max is only moved when it grows by more than
// 2^8 (values of P stay <= 256), so O in TMEM is rescaled rarely.
//
// Causal semantics (gqa_kernels/gqa_fwd.py:70-73, :94-96): the key loop of a
// CTA ends at the last key any of its rows can see; row r masks keys beyond
// its own position + (seq_kv - seq_q). Only the last one or two key tiles of a
// CTA need the mask.
//
// Paged K/V (PAGED): K and V come from vLLM-layout block caches. The producer
// loads each 128-key tile as two 64-key boxes, each from the physical block the
// sequence's block table names; a box past the sequence's end gets an
// out-of-range block coordinate, so TMA fills it with zeros. Each sequence has
// its own length (read after the grid dependency wait) and so its own causal
// offset; the tile plan is made for the host's bound of the lengths.
#pragma once

#include "gqa_common.cuh"

namespace gqa {

struct PrefillParams {
  int batch, hq, hkv, group, seq_q, seq_kv;
  int bm;       // positions per tile = 128 / group
  int n_pairs;  // ceil(ceil(seq_q / bm) / 2)
  // Unit order. Pair-major (unit_inner = batch * hkv): the longest query pairs of all
  // (batch, kv head) first, which balances causal work. Head-major (unit_inner =
  // n_pairs): the pairs of one (batch, kv head) side by side, so the CTAs reading the
  // same keys and values run together and share them in L2; the host picks it when
  // the pairs' key counts are within a factor of two.
  int head_major;
  int unit_inner;
  int causal;
  float scale_log2;
  // Key-axis split of each unit (query pair of one (batch, kv head)) across
  // nsplit CTAs of chunk_tiles key tiles each; 1 = no split. Split CTAs publish
  // fp32 partials m, l [unit][split][256 rows] and acc [unit][split][HD][256 rows]
  // (row fastest, so a warp's accesses coalesce), and the last CTA of the
  // unit (atomic ticket ws_cnt[unit], zero between calls) combines them.
  int nsplit;
  int chunk_tiles;
  float* ws_m;
  float* ws_l;
  float* ws_acc;
  unsigned* ws_cnt;
  // Paged K/V (the PAGED instantiation): the caches are [num_blocks][block_size][hkv][HD];
  // key k of sequence b sits in physical block block_table[b * bt_stride + (k >> block_shift)]
  // at position k & (block_size - 1), and the sequence holds min(seq_lens[b], seq_kv) keys
  // (seq_kv is then the host's bound of the lengths). Query position i of sequence b is
  // key position len_b - seq_q + i (bottom-right alignment per sequence).
  const int* block_table;
  const int* seq_lens;
  int bt_stride;
  int block_shift;
  int num_blocks;
};

// Work item of CTA `cta`: unit = (query pair, batch, kv head) in the order above,
// longest pair of a head first; split = which chunk of the unit's key tiles. A unit with fewer key tiles than
// the splits cover uses fewer splits (n_valid); the others return at once.
struct PrefillWork {
  int unit, split, n_valid, b, kvh, p0, j0, nk;
};

template <int BN, bool SPLIT>
__device__ __forceinline__ PrefillWork prefill_work(const PrefillParams& p, unsigned cta) {
  // The integer forms below (unsigned division of the CTA index, signed after it)
  // are the ones under which the unsplit instantiation compiles without register
  // spills at the 208-register softmax budget; recheck `-Xptxas -v` after changes.
  PrefillWork w;
  const unsigned unit = SPLIT ? cta / (unsigned)p.nsplit : cta;
  w.split = SPLIT ? (int)(cta % (unsigned)p.nsplit) : 0;
  w.unit = (int)unit;
  const int inner = unit % p.unit_inner;
  const int outer = unit / p.unit_inner;
  const int bh = p.head_major ? outer : inner;
  const int pair = p.n_pairs - 1 - (p.head_major ? inner : outer);
  w.b = bh / p.hkv;
  w.kvh = bh % p.hkv;
  w.p0 = pair * 2 * p.bm;  // first position of tile 0
  const int off = p.seq_kv - p.seq_q;
  int kv_end = p.seq_kv;
  if (p.causal) kv_end = min(kv_end, min(w.p0 + 2 * p.bm, p.seq_q) + off);
  const int nk_unit = (kv_end > 0) ? (kv_end + BN - 1) / BN : 0;
  w.n_valid = SPLIT ? max(1, (nk_unit + p.chunk_tiles - 1) / p.chunk_tiles) : 1;
  w.j0 = (SPLIT && w.n_valid > 1) ? w.split * p.chunk_tiles : 0;  // key tiles [j0, j0 + nk)
  w.nk = (SPLIT && w.n_valid > 1) ? min(nk_unit, w.j0 + p.chunk_tiles) - w.j0 : nk_unit;
  return w;
}

// Key tiles of a paged work item once its sequence's length kv_len is known. The
// plan (n_valid, j0) was made for the host's bound seq_kv; a split past a shorter
// sequence's last tile gets none and publishes an empty partial.
template <int BN>
__device__ __forceinline__ int paged_work_tiles(const PrefillParams& p, const PrefillWork& w, int kv_len) {
  int kv_end = kv_len;
  if (p.causal) kv_end = min(kv_end, min(w.p0 + 2 * p.bm, p.seq_q) + kv_len - p.seq_q);
  const int nk_unit = (kv_end > 0) ? (kv_end + BN - 1) / BN : 0;
  if (w.n_valid > 1) return max(0, min(nk_unit, w.j0 + p.chunk_tiles) - w.j0);
  return nk_unit;
}

template <int HD>
struct PrefillCfg {
  static constexpr int kRows = 128;                  // packed rows per query tile (UMMA M)
  static constexpr int kBN = 128;                    // keys per tile (UMMA N of S, K of PV)
  static constexpr int kNSub = HD / 64;              // 128-byte swizzle sub-tiles along d
  static constexpr int kSubBytes = 128 * 128;        // 128 rows x 128 B
  static constexpr int kTileBytes = kNSub * kSubBytes;  // one Q, K or V tile
  static constexpr int kSlots = (HD == 128) ? 4 : 8;    // K/V ring slots (K and V alternate)
  static constexpr int kQOff = 0;
  static constexpr int kKVOff = 2 * kTileBytes;
  static constexpr int kBarOff = kKVOff + kSlots * kTileBytes;
  // P is published to the MMA warp in kPParts column parts per tile, each with its own
  // barrier, so the PV UMMAs of a part start while the next part is computed.
  static constexpr int kPParts = 2;
  // barriers: q_full[2] kv_full[S] kv_empty[S] s_full[2] p_full[2 tiles][kPParts] o_final[2] mma_done
  static constexpr int kNumBars = 2 + 2 * kSlots + 2 + 2 * kPParts + 2 + 1;
  // tmem base, abort flag, last-CTA flag, paged key tiles, paged sequence length
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kMiscOff + 32 + 1024;  // + alignment slack
  // warps 0-3 softmax tile 0, 4-7 softmax tile 1, 8 MMA issuer, 9 TMA producer, 10-11 idle
  static constexpr int kThreads = 384;
  static constexpr int kTmemCols = 512;
  // setmaxnreg split. The launch holds kThreads x (registers per thread at launch)
  // registers; the split needs 2 x 128 x kSoftmaxRegs + 128 x kControlRegs of them.
  // gqa_sm100.cu checks the compiled register count before every launch.
  static constexpr int kSoftmaxRegs = 208;
  static constexpr int kControlRegs = 88;
  static constexpr int kRegsNeeded = 256 * kSoftmaxRegs + 128 * kControlRegs;  // 64512 = 384 x 168
  static constexpr int kColS0 = 0, kColS1 = 128, kColO0 = 256, kColO1 = 256 + HD;
  // Of every eight column pairs of P, this many take the MUFU ex2 and the rest the
  // polynomial exp2 on the FMA pipe (exp2_poly2). Measured on B200 (8K causal
  // prefill): 7 of 8 472 us, 8 of 8 473 us, 6 of 8 490 us, 5 of 8 514 us.
  static constexpr int kMufuPairsPer8 = 7;
};

template <int HD, bool BF16, bool SPLIT, bool PAGED = false>
__global__ void __launch_bounds__(384, 1)
    gqa_prefill_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap qmap,
                       const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                       const __grid_constant__ CUtensorMap omap) {
  using Cfg = PrefillCfg<HD>;
  constexpr int NSUB = Cfg::kNSub;
  constexpr int SLOTS = Cfg::kSlots;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* const smem = smem_raw + (base - raw_base);

  const uint32_t q_smem0 = base + Cfg::kQOff;
  const uint32_t kv_smem0 = base + Cfg::kKVOff;
  const uint32_t bars = base + Cfg::kBarOff;
  const uint32_t bar_q_full = bars;                      // [2]
  const uint32_t bar_kv_full = bars + 16;                // [SLOTS]
  const uint32_t bar_kv_empty = bar_kv_full + 8 * SLOTS; // [SLOTS]
  const uint32_t bar_s_full = bar_kv_empty + 8 * SLOTS;  // [2]
  const uint32_t bar_p_full = bar_s_full + 16;           // [2][kPParts]: (tile, column part of P)
  const uint32_t bar_o_final = bar_p_full + 16 * Cfg::kPParts;  // [2]
  const uint32_t bar_mma_done = bar_o_final + 16;
  uint32_t* tmem_base_ptr = reinterpret_cast<uint32_t*>(smem + Cfg::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kMiscOff + 4);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  // ---- work item: longest (highest) query pair first, across all (b, kv) ----
  const PrefillWork wk = prefill_work<Cfg::kBN, SPLIT>(p, blockIdx.x);
  if (wk.split >= wk.n_valid) return;  // whole CTA, before any barrier or TMEM use
  const int b = wk.b, kvh = wk.kvh, p0 = wk.p0, j0 = wk.j0;
  // A paged CTA's key tiles and sequence length depend on a value read from global
  // memory; they are kept in shared memory (written by thread 0 before the CTA
  // barrier below) and read where used, rather than held in registers across the
  // loops: the softmax warps have none to spare, and the dense values are
  // recomputed from parameters instead.
  volatile int* const paged_info = reinterpret_cast<volatile int*>(smem + Cfg::kMiscOff + 12);
  auto work_tiles = [&]() -> int {
    if constexpr (PAGED) return paged_info[0]; else return wk.nk;
  };
  auto seq_len = [&]() -> int {
    if constexpr (PAGED) return paged_info[1]; else return p.seq_kv;
  };

  if (tid == 0) {
    mbar_init(bar_q_full, 1);
    mbar_init(bar_q_full + 8, 1);
    for (int s = 0; s < SLOTS; ++s) {
      mbar_init(bar_kv_full + 8 * s, 1);
      mbar_init(bar_kv_empty + 8 * s, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_s_full + 8 * i, 1);
      for (int h = 0; h < Cfg::kPParts; ++h) mbar_init(bar_p_full + 8 * (Cfg::kPParts * i + h), 128);
      mbar_init(bar_o_final + 8 * i, 1);
    }
    mbar_init(bar_mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  // Before any global memory access and before taking TMEM, the previous grid on
  // the stream has finished (programmatic dependent launch).
  pdl_wait();
  pdl_trigger();
  if constexpr (PAGED) {
    if (tid == 0) {
      // A length above the host's bound is clipped to it (the plan covers seq_kv keys);
      // the checked build reports such a call.
      (void)GQA_CHECK(p.seq_lens[b] <= p.seq_kv, 906);
      const int len = max(0, min(p.seq_lens[b], p.seq_kv));
      paged_info[1] = len;
      paged_info[0] = paged_work_tiles<Cfg::kBN>(p, wk, len);
    }
  }
  if (warp == 8) {
    tmem_alloc(smem_u32(tmem_base_ptr), Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_ptr;

  // Register split: 2 x 208 (softmax warpgroups) + 88 (control warpgroup) = 504 per thread-slot,
  // i.e. 64512 registers = the 384 x 168 the kernel is launched with.
  static_assert(Cfg::kSoftmaxRegs == 208 && Cfg::kControlRegs == 88, "keep the asm immediates in sync");
  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 88;" ::: "memory");
  if (warp == 9) {
    // ================================================================ producer
    const int nk = work_tiles();
    const int kv_len = seq_len();
    if (lane == 0 && nk > 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      const int hq0 = kvh * p.group;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        mbar_arrive_expect_tx(bar_q_full + 8 * i, Cfg::kTileBytes);
#pragma unroll
        for (int s = 0; s < NSUB; ++s)
          tma_load_4d(q_smem0 + i * Cfg::kTileBytes + s * Cfg::kSubBytes, &qmap, bar_q_full + 8 * i, s * 64,
                      p0 + i * p.bm, hq0, b);
      }
      int t = 0;
      const int n_loads = 2 * nk;
      int pb0 = 0, pb1 = 0;  // paged: physical blocks of the tile's two 64-key boxes
      for (; t < n_loads; ++t) {
        const int slot = t % SLOTS;
        const int use = t / SLOTS;
        const int key0 = (j0 + (t >> 1)) * Cfg::kBN;
        if constexpr (PAGED) {
          // Looked up once per tile (K loads; V reuses them) and before the slot
          // wait, so the table read overlaps it.
          if ((t & 1) == 0) {
            const int* row_bt = p.block_table + (int64_t)b * p.bt_stride;
            pb0 = (key0 < kv_len) ? row_bt[key0 >> p.block_shift] : p.num_blocks;
            pb1 = (key0 + 64 < kv_len) ? row_bt[(key0 + 64) >> p.block_shift] : p.num_blocks;
          }
        }
        if (use > 0 && !mbar_wait(bar_kv_empty + 8 * slot, (use - 1) & 1, abort_flag, 1)) break;
        if (withheld_load(t)) continue;
        const uint32_t full = bar_kv_full + 8 * slot;
        mbar_arrive_expect_tx(full, Cfg::kTileBytes);
        const CUtensorMap* map = (t & 1) ? &vmap : &kmap;
        if constexpr (PAGED) {
          // Map (d, kv head, position in block, block), box {64, 1, 64, 1}: 64 rows of
          // 128 bytes, so the two boxes of a sub-tile form its 128 swizzled rows.
          const int pos0 = key0 & ((1 << p.block_shift) - 1);
#pragma unroll
          for (int s = 0; s < NSUB; ++s) {
            const uint32_t dst = kv_smem0 + slot * Cfg::kTileBytes + s * Cfg::kSubBytes;
            tma_load_4d(dst, map, full, s * 64, kvh, pos0, pb0);
            tma_load_4d(dst + Cfg::kSubBytes / 2, map, full, s * 64, kvh,
                        (key0 + 64) & ((1 << p.block_shift) - 1), pb1);
          }
        } else {
#pragma unroll
          for (int s = 0; s < NSUB; ++s)
            tma_load_4d(kv_smem0 + slot * Cfg::kTileBytes + s * Cfg::kSubBytes, map, full, s * 64, key0, kvh, b);
        }
      }
      if (t < n_loads) {  // aborted: let in-flight loads land before teardown
        volatile int dummy = 0;
        for (int u = max(0, t - SLOTS); u < t; ++u)
          if (!withheld_load(u)) mbar_wait(bar_kv_full + 8 * (u % SLOTS), (u / SLOTS) & 1, &dummy, 2);
      }
    }
  } else if (warp == 8) {
    // ================================================================ MMA issuer
    const int nk = work_tiles();
    if (lane == 0 && nk > 0) {
      constexpr uint32_t idesc_qk = make_idesc_f16(128, Cfg::kBN, BF16, false);
      constexpr uint32_t idesc_pv = make_idesc_f16(128, HD, BF16, true);
      auto issue_qk = [&](int i, int slot) {
        const uint32_t tS = tmem_base + (i ? Cfg::kColS1 : Cfg::kColS0);
        const uint32_t qa = q_smem0 + i * Cfg::kTileBytes;
        const uint32_t kb = kv_smem0 + slot * Cfg::kTileBytes;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t o = (k >> 2) * Cfg::kSubBytes + (k & 3) * 32;
          umma_ss(tS, desc_sw128_kmajor(qa + o), desc_sw128_kmajor(kb + o), idesc_qk, k > 0 ? 1u : 0u);
        }
      };
      // O_i += P_i V over column part h of the tile (UMMAs of 16 keys each).
      auto issue_pv = [&](int i, int slot, int h, bool acc) {
        const uint32_t tS = tmem_base + (i ? Cfg::kColS1 : Cfg::kColS0);
        const uint32_t tO = tmem_base + (i ? Cfg::kColO1 : Cfg::kColO0);
        const uint32_t vb = kv_smem0 + slot * Cfg::kTileBytes;
        constexpr int kPerPart = Cfg::kBN / 16 / Cfg::kPParts;
#pragma unroll
        for (int kk = 0; kk < kPerPart; ++kk) {
          const int k = h * kPerPart + kk;
          // P: 16 keys = 8 TMEM columns of packed 16-bit pairs; V: 16 key rows of 128 B.
          umma_ts(tO, tS + k * 8, desc_sw128_mnmajor(vb + k * 16 * 128, Cfg::kSubBytes), idesc_pv,
                  (acc || k > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(bar_q_full, 0, abort_flag, 10) && mbar_wait(bar_q_full + 8, 0, abort_flag, 11) &&
                mbar_wait(bar_kv_full, 0, abort_flag, 12);
      if (ok) {
        tc_fence_after();
        issue_qk(0, 0);
        umma_commit(bar_s_full);
        issue_qk(1, 0);
        umma_commit(bar_s_full + 8);
        umma_commit(bar_kv_empty);  // K_0 consumed
        for (int j = 0; j < nk; ++j) {
          const int tv = 2 * j + 1, sv = tv % SLOTS;
          const int tk = 2 * j + 2, sk = tk % SLOTS;
          if (!mbar_wait(bar_kv_full + 8 * sv, (tv / SLOTS) & 1, abort_flag, 13)) break;
          bool pv_ok = true;
#pragma unroll
          for (int h = 0; h < Cfg::kPParts && pv_ok; ++h) {
            pv_ok = mbar_wait(bar_p_full + 8 * h, j & 1, abort_flag, h ? 18 : 14);
            if (pv_ok) {
              tc_fence_after();
              issue_pv(0, sv, h, h > 0 || j > 0);
            }
          }
          if (!pv_ok) break;
          const bool more = (j + 1 < nk);
          if (more) {
            if (!mbar_wait(bar_kv_full + 8 * sk, (tk / SLOTS) & 1, abort_flag, 15)) break;
            tc_fence_after();
            issue_qk(0, sk);
            umma_commit(bar_s_full);
          } else {
            umma_commit(bar_o_final);
          }
#pragma unroll
          for (int h = 0; h < Cfg::kPParts && pv_ok; ++h) {
            pv_ok = mbar_wait(bar_p_full + 8 * (Cfg::kPParts + h), j & 1, abort_flag, h ? 19 : 16);
            if (pv_ok) {
              tc_fence_after();
              issue_pv(1, sv, h, h > 0 || j > 0);
            }
          }
          if (!pv_ok) break;
          umma_commit(bar_kv_empty + 8 * sv);  // V_j consumed
          if (more) {
            issue_qk(1, sk);
            umma_commit(bar_s_full + 8);
            umma_commit(bar_kv_empty + 8 * sk);  // K_{j+1} consumed
          } else {
            umma_commit(bar_o_final + 8);
          }
        }
      }
      // Drain: every MMA issued above completes before TMEM is released.
      umma_commit(bar_mma_done);
      volatile int dummy = 0;
      mbar_wait(bar_mma_done, 0, &dummy, 17);
    }
    __syncwarp();
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 208;" ::: "memory");
    // ================================================================ softmax warpgroups
    const int wg = warp >> 2;    // query tile handled by this warpgroup
    const int row = tid & 127;   // packed row == TMEM lane
    const int wq = warp & 3;     // TMEM lane quarter of this warp
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem_base + lane_off + (wg ? Cfg::kColS1 : Cfg::kColS0);
    const uint32_t tO = tmem_base + lane_off + (wg ? Cfg::kColO1 : Cfg::kColO0);
    const uint32_t s_full = bar_s_full + 8 * wg;
    const uint32_t p_full = bar_p_full + 8 * Cfg::kPParts * wg;  // + 8 per column part

    const int g = row / p.bm;
    const int pos = p0 + wg * p.bm + (row - g * p.bm);
    // Number of keys this row may see, counted from this CTA's first key tile.
    auto row_lim = [&]() -> int {
      const int len = seq_len();
      const int lim = p.causal ? min(len, pos + len - p.seq_q + 1) : len;
      return lim - j0 * Cfg::kBN;
    };
    const float scale = p.scale_log2;

    // A row that sees no key at all keeps m = -inf, and its NaN (exp2(-inf + inf))
    // reaches the output, as in the reference. Such rows only occur in units of at
    // most two key tiles, which are never split (paged sequences shorter than the
    // plan's bound excepted: the combine marks them). In a split unit a row may see no
    // key of this CTA's chunk while it sees keys of others: a finite start value
    // keeps its P finite (exp2(-inf + 3e38) = 0), and the combine gives the chunk
    // the weight exp2(-3e38 - M) = 0.
    float m_run = (wk.n_valid > 1) ? -3.0e38f : -INFINITY;
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < work_tiles(); ++j) {
      ok = mbar_wait(s_full, j & 1, abort_flag, 20 + wg);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      if constexpr (PAGED) {
        // The tile holding the sequence's end: its keys past the end are masked (P = 0),
        // but the cache block's stale slots there may hold NaN or Inf, and 0 x NaN would
        // reach O through the PV MMA. Once V has landed, each thread zeroes its row of V
        // if that key is past the end (both warpgroups write the same zeros), then fences
        // the generic writes against the MMA's reads before P is published.
        const int nv = seq_len() - (j0 + j) * Cfg::kBN;
        if (nv < Cfg::kBN) {
          const int tv = 2 * j + 1;
          ok = mbar_wait(bar_kv_full + 8 * (tv % SLOTS), (tv / SLOTS) & 1, abort_flag, 24 + wg);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          if (row >= nv) {
            const uint32_t vrow = kv_smem0 + (tv % SLOTS) * Cfg::kTileBytes + row * 128;
#pragma unroll
            for (int c = 0; c < NSUB * 8; ++c)
              asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(vrow + (c >> 3) * Cfg::kSubBytes +
                                                                          (c & 7) * 16),
                           "r"(0u)
                           : "memory");
          }
          fence_proxy_async_smem();
        }
      }
      // S row: the second half's TMEM load is in flight while the first half's max
      // is computed (the partial maxima feed the second wait, so they precede it).
      uint32_t sr[128];
      tmem_ld32(tS + 0, sr + 0);
      tmem_ld32(tS + 32, sr + 32);
      tmem_wait_ld();
      reg_fence_n<64>(sr);
      tmem_ld32(tS + 64, sr + 64);
      tmem_ld32(tS + 96, sr + 96);
      const int rem = row_lim() - j * Cfg::kBN;  // visible columns in this tile
      const bool masked = rem < Cfg::kBN;
      if (masked) {
#pragma unroll
        for (int c = 0; c < 64; ++c) sr[c] = (c < rem) ? sr[c] : __float_as_uint(-INFINITY);
      }
      // Row max with three-input maxima, four independent chains.
      float mx0 = __uint_as_float(sr[0]), mx1 = __uint_as_float(sr[1]);
      float mx2 = __uint_as_float(sr[2]), mx3 = __uint_as_float(sr[3]);
#pragma unroll
      for (int c = 4; c < 60; c += 8) {
        mx0 = max3(mx0, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
        mx1 = max3(mx1, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
        mx2 = max3(mx2, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
        mx3 = max3(mx3, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
      }
      mx0 = max3(mx0, __uint_as_float(sr[60]), __uint_as_float(sr[61]));
      mx1 = max3(mx1, __uint_as_float(sr[62]), __uint_as_float(sr[63]));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::"f"(mx0), "f"(mx1), "f"(mx2), "f"(mx3) : "memory");
      reg_fence_n<64>(sr + 64);
      if (masked) {
#pragma unroll
        for (int c = 64; c < 128; ++c) sr[c] = (c < rem) ? sr[c] : __float_as_uint(-INFINITY);
      }
#pragma unroll
      for (int c = 64; c < 128; c += 8) {
        mx0 = max3(mx0, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
        mx1 = max3(mx1, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
        mx2 = max3(mx2, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
        mx3 = max3(mx3, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
      }
      const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * scale;
      const float m_new = fmaxf(m_run, mx);
      const bool need = m_new > m_run + 8.0f;  // false while both are -inf
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        const float alpha = need ? fast_exp2(m_run - m_new) : 1.0f;
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t orr[32];
          tmem_ld32(tO + c * 32, orr);
          tmem_wait_ld();
          reg_fence(orr);
#pragma unroll
          for (int e = 0; e < 32; ++e) orr[e] = __float_as_uint(__uint_as_float(orr[e]) * alpha);
          tmem_st32(tO + c * 32, orr);
        }
        tmem_wait_st();
      }
      if (need) {
        l_run *= fast_exp2(m_run - m_new);
        m_run = m_new;
      }
      // P = exp2(S * scale - m), written over S as packed 16-bit pairs, in kPParts column
      // parts so the PV MMAs of a part start while the next one is computed.
      // One column pair in eight takes the polynomial exp2 on the FMA pipe, the rest
      // the MUFU ex2; the row sum and the scale use packed two-lane fp32 math.
      const float2 sc2 = make_float2(scale, scale);
      const float2 nm2 = make_float2(-m_run, -m_run);
      float2 sum2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      constexpr int kPairs = 64 / Cfg::kPParts;  // column pairs (packed TMEM columns) per part
#pragma unroll
      for (int h = 0; h < Cfg::kPParts; ++h) {
        uint32_t pk[kPairs];
#pragma unroll
        for (int c = 0; c < kPairs; ++c) {
          const int col = 2 * kPairs * h + 2 * c;
          const float2 x = fma2(make_float2(__uint_as_float(sr[col]), __uint_as_float(sr[col + 1])), sc2, nm2);
          float2 pv;
          if ((c & 7) >= Cfg::kMufuPairsPer8) {
            pv = exp2_poly2(x);
          } else {
            pv.x = fast_exp2(x.x);
            pv.y = fast_exp2(x.y);
          }
          sum2[c & 3] = add2(sum2[c & 3], pv);
          pk[c] = pack2<BF16>(pv.x, pv.y);
        }
        if constexpr (kPairs >= 32) {
#pragma unroll
          for (int q = 0; q < kPairs / 32; ++q) tmem_st32(tS + kPairs * h + 32 * q, pk + 32 * q);
        } else {
          tmem_st16(tS + 16 * h, pk);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(p_full + 8 * h);
      }
      const float2 s01 = add2(sum2[0], sum2[1]);
      const float2 s23 = add2(sum2[2], sum2[3]);
      const float2 st = add2(s01, s23);
      l_run += st.x + st.y;
    }

    // ---- epilogue: O / l -> 16-bit -> swizzled staging (this tile's Q buffer) -> TMA store
    bool have_o = ok && work_tiles() > 0;
    if (have_o) {
      have_o = mbar_wait(bar_o_final + 8 * wg, 0, abort_flag, 22 + wg);
      have_o = __all_sync(0xffffffffu, have_o);
    }
    if (have_o) tc_fence_after();

    // Key-split unit: publish this CTA's partial; the last CTA of the unit folds
    // the other splits' partials into its own before the store below. The work item
    // is derived again from a fresh read of the CTA index, so none of its fields
    // stays live in registers across the softmax loop.
    int unit = 0, split = 0, n_valid = 1;
    if constexpr (SPLIT) {
      unsigned cta;
      asm volatile("mov.u32 %0, %%ctaid.x;" : "=r"(cta));
      const PrefillWork wk2 = prefill_work<Cfg::kBN, SPLIT>(p, cta);
      unit = wk2.unit;
      split = wk2.split;
      n_valid = wk2.n_valid;
    }
    float inv = 1.0f / l_run;  // l == 0 -> inf -> NaN rows, the reference's 0/0
    float m_ref = 0.f;                       // reference max of the combined splits
    bool store = true;
    int n_other = 0;
    // Partials of the unit: m, l [split][256 rows] and acc [split][d][256 rows]; a
    // warp's 32 rows are consecutive, so every access below is one 128-byte line.
    const int prow = wg * 128 + row;  // row of the unit's 256 packed rows
    const int64_t pbase = ((int64_t)unit * p.nsplit) * 256 + prow;
    if (n_valid > 1) {
      __stcg(p.ws_m + pbase + (int64_t)split * 256, m_run);
      __stcg(p.ws_l + pbase + (int64_t)split * 256, l_run);
      float* acc_own = p.ws_acc + ((int64_t)unit * p.nsplit + split) * HD * 256 + prow;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t orr[32];
        if (have_o) {
          tmem_ld32(tO + c * 32, orr);
          tmem_wait_ld();
          reg_fence(orr);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) orr[e] = (PAGED && work_tiles() == 0) ? 0u : 0x7fc00000u;  // empty split: 0
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) __stcg(acc_own + (c * 32 + e) * 256, __uint_as_float(orr[e]));
      }
      // Both softmax warpgroups have published; thread 0's release-acquire ticket
      // (fences are cumulative) tells whether this CTA is the unit's last.
      asm volatile("bar.sync 3, 256;" ::: "memory");
      uint32_t* last_slot = tmem_base_ptr + 2;
      if (tid == 0) {
        unsigned ticket;
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(ticket) : "l"(p.ws_cnt + unit)
                     : "memory");
        const bool last = ticket == (unsigned)(n_valid - 1);
        *last_slot = last ? 1u : 0u;
        if (last) p.ws_cnt[unit] = 0u;  // every split has arrived: ready for the next call
      }
      asm volatile("bar.sync 3, 256;" ::: "memory");
      store = *last_slot != 0;
      if (store) {
        // Combined weights of this row over the splits: w_s = exp2(m_s - max m). The
        // other splits' m and l are read four at a time (clamped indices, own split
        // and indices past the last masked out) so their latencies overlap.
        float M = m_run;
        for (int s0 = 0; s0 < n_valid; s0 += 4) {
          float mv[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) mv[i] = __ldcg(p.ws_m + pbase + (int64_t)min(s0 + i, n_valid - 1) * 256);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (s0 + i < n_valid && s0 + i != split) M = fmaxf(M, mv[i]);
        }
        const float Mu = (M == -INFINITY) ? 0.f : M;
        // L = sum over splits in split order (this CTA's own terms from registers, the
        // same values it published), so the result does not depend on which CTA of the
        // unit arrives last.
        float L = 0.f;
        for (int s0 = 0; s0 < n_valid; s0 += 4) {
          float mv[4], lv[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int64_t o2 = pbase + (int64_t)min(s0 + i, n_valid - 1) * 256;
            mv[i] = __ldcg(p.ws_m + o2);
            lv[i] = __ldcg(p.ws_l + o2);
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (s0 + i >= n_valid) continue;
            const bool own = s0 + i == split;
            L += fast_exp2((own ? m_run : mv[i]) - Mu) * (own ? l_run : lv[i]);
          }
        }
        inv = 1.0f / L;
        if constexpr (PAGED) {
          // A paged sequence shorter than the chunk has rows that see no key in any
          // split (every m still at its start value): NaN, as in the reference.
          if (M == -3.0e38f) inv = __int_as_float(0x7fc00000);
        }
        n_other = n_valid - 1;
        m_ref = Mu;
      }
    }
    const uint32_t stage = q_smem0 + wg * Cfg::kTileBytes;
#pragma unroll
    for (int c = 0; c < HD / 32; ++c) {
      uint32_t orr[32];
      if (have_o) {
        tmem_ld32(tO + c * 32, orr);
        tmem_wait_ld();
        reg_fence(orr);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) orr[e] = (PAGED && work_tiles() == 0) ? 0u : 0x7fc00000u;  // empty split: 0
      }
      if (n_other > 0) {
        // Fold the splits in split order, two per pass (64 independent loads in flight
        // per thread); this CTA's own split comes from its TMEM values. An index past
        // the last split reads a valid partial at weight 0.
        uint32_t own[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          own[e] = orr[e];
          orr[e] = 0u;
        }
        for (int s0 = 0; s0 < n_valid; s0 += 2) {
          const int sa = s0, sb = min(s0 + 1, n_valid - 1);
          const float ma = (sa == split) ? m_run : __ldcg(p.ws_m + pbase + (int64_t)sa * 256);
          const float mb = (sb == split) ? m_run : __ldcg(p.ws_m + pbase + (int64_t)sb * 256);
          const float wa = fast_exp2(ma - m_ref);
          const float wb = (s0 + 1 >= n_valid) ? 0.f : fast_exp2(mb - m_ref);
          const float* xa = p.ws_acc + ((int64_t)unit * p.nsplit + sa) * HD * 256 + prow + c * 32 * 256;
          const float* xb = p.ws_acc + ((int64_t)unit * p.nsplit + sb) * HD * 256 + prow + c * 32 * 256;
          float va[32], vb[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            va[e] = (sa == split) ? __uint_as_float(own[e]) : __ldcg(xa + e * 256);
            vb[e] = (sb == split) ? __uint_as_float(own[e]) : __ldcg(xb + e * 256);
          }
#pragma unroll
          for (int e = 0; e < 32; ++e)
            orr[e] = __float_as_uint(fmaf(wb, vb[e], fmaf(wa, va[e], __uint_as_float(orr[e]))));
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int chunk = 4 * c + e;  // 16-byte chunk along d (8 values)
#define GQA_OV(i) (__uint_as_float(orr[8 * e + (i)]) * inv)
        const uint32_t w0 = pack2<BF16>(GQA_OV(0), GQA_OV(1));
        const uint32_t w1 = pack2<BF16>(GQA_OV(2), GQA_OV(3));
        const uint32_t w2 = pack2<BF16>(GQA_OV(4), GQA_OV(5));
        const uint32_t w3 = pack2<BF16>(GQA_OV(6), GQA_OV(7));
#undef GQA_OV
        const uint32_t dst = stage + (chunk >> 3) * Cfg::kSubBytes + sw128_off(row, chunk & 7);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(w0), "r"(w1), "r"(w2), "r"(w3)
                     : "memory");
      }
    }
    fence_proxy_async_smem();
    if (wg == 0)
      asm volatile("bar.sync 1, 128;" ::: "memory");
    else
      asm volatile("bar.sync 2, 128;" ::: "memory");
    const int tile_pos = p0 + wg * p.bm;
    if (store && row == 0 && tile_pos < p.seq_q) {
#pragma unroll
      for (int s = 0; s < NSUB; ++s)
        tma_store_4d(&omap, stage + s * Cfg::kSubBytes, s * 64, tile_pos, kvh * p.group, b);
      bulk_commit_group();
      bulk_wait_group0();
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 8) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

}  // namespace gqa
