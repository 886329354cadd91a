// HBM-streaming GQA attention kernel for few packed query rows (decode,
// short chunked prefill). One CTA streams one chunk of the key axis of one
// (batch, kv_head, q-block) unit through a TMA ring and keeps the online
// softmax state of up to 64 packed rows (group_size heads x block_m positions)
// in mma.sync accumulators. At <= 64 rows per 512 bytes of K+V the kernel is
// bound by HBM bandwidth, not by the tensor pipe; what matters is keeping
// enough bytes in flight (a 192 KB ring, one CTA per SM) and enough warps
// (eight compute warps, two per SM sub-partition) to hide the MMA/shuffle
// latency of each stage behind the next stage's arrival.
//
// Reference behaviour followed:
//   gqa_kernels/gqa_split.py:46-112   per-chunk partial (m, l, acc), causal chunk clip
//   gqa_kernels/gqa_split.py:134-147  log-sum-exp combine (fused here: last CTA per unit)
//   gqa_kernels/gqa_fwd.py:57-73      group packing, bottom-right causal offset
#pragma once

#include "gqa_common.cuh"

namespace gqa {

enum StreamMode : int {
  kStreamOut = 0,           // nsplit == 1: write O directly
  kStreamRefPartial = 1,    // write (m, l, acc) at split index into caller arrays (reference layout)
  kStreamFused = 2,         // write partial to workspace; last CTA of the unit combines into O
  kStreamFusedPartial = 3,  // as kStreamFused, but the last CTA writes the combined (m, l, acc)
};

struct StreamParams {
  const uint16_t* q;
  void* o;
  int64_t q_sb, q_sh, q_sm;  // element strides of Q (d stride is 1)
  int64_t o_sb, o_sh, o_sm;
  int batch, hq, hkv, group, seq_q, seq_kv;  // seq_kv: keys held by k/v (local shard)
  int block_m;    // query positions per unit
  int n_mtiles;   // ceil(seq_q / block_m)
  int rows;       // group * block_m packed rows per unit (<= 16 * RG)
  int nsplit;     // chunks per unit (gridDim.x = units * nsplit)
  int chunk;      // keys per chunk (a multiple of 64, or the reference's chunk size)
  int causal;
  float scale_log2;
  int kv_offset;     // global position of local key 0
  int seq_kv_total;  // global key count (causal offset = seq_kv_total - seq_q)
  int mode;
  // kStreamRefPartial outputs
  float* m_p;
  float* l_p;
  float* acc_p;
  int64_t p_sb, p_sh, p_sm, p_ss;
  int64_t a_sb, a_sh, a_sm, a_ss, a_sd;
  // kStreamFused / kStreamFusedPartial workspace
  float* ws_m;    // [units][nsplit][rows]
  float* ws_l;    // [units][nsplit][rows]
  float* ws_acc;  // [units][nsplit][rows][HD]
  unsigned* ws_cnt;  // [units] ticket counters, zero between calls
  // kStreamFusedPartial outputs, contiguous (batch, hq, seq_q[, HD])
  float* m_out;
  float* l_out;
  float* acc_out;
  // Paged K/V (block_table != nullptr): the caches are [num_blocks][block_size][hkv][HD]
  // (the K/V tensor maps are (HD, hkv, block_size, num_blocks)); sequence b's key k lives
  // in physical block block_table[b * bt_stride + (k >> block_shift)] at position
  // k & (block_size - 1), and the sequence holds seq_lens[b] keys. block_size is a power
  // of two >= 64, so a 64-key box never crosses a block. The sequence's seq_q queries
  // are its last seq_q positions (causal offset seq_lens[b] - seq_q).
  const int* block_table;
  const int* seq_lens;
  int bt_stride;
  int block_shift;
  // fp8 K/V (the FP8 instantiation): stored value x scale = real value. k_scale is
  // folded into scale_log2 by the host; v_scale multiplies the accumulators once.
  float v_scale;
  // Peer exchange (kStreamFusedPartial with npeer > 0, the key-sharded multi-GPU
  // combine): the unit's combined (m, l, acc) goes to slot my_rank of every rank's
  // receive buffer -- plain stores, over NVLink for the other ranks -- in the packed
  // layout [m | l | pad | acc] (l at pk_rows, acc at pk_acc floats), into the parity
  // (*epoch & 1) half. After the stores, one system-scope release add per rank on
  // that rank's counter for this source: the ranks' combines wait for it.
  float* peer_base[kMaxPeers];              // each rank's receive buffer, parity 0 slot 0
  unsigned long long* peer_cnt[kMaxPeers];  // each rank's counters [world], one per source
  const unsigned long long* epoch;          // this rank's call counter (gqa_epoch_bump)
  int64_t peer_slot, peer_parity;           // floats per source slot, per parity half
  int64_t pk_rows, pk_acc;
  int npeer, my_rank;
};

template <int HD>
struct StreamCfg {
  static constexpr int kBN = 128;                      // keys per stage
  static constexpr int kBox = 64;                      // keys per TMA box
  static constexpr int kNSub = HD / 64;                // 128-byte swizzle sub-tiles along d
  static constexpr int kSubBytes = kBN * 128;          // one d sub-tile over the stage's keys
  static constexpr int kBoxBytes = kBox * 128;         // one TMA box
  static constexpr int kTileBytes = kNSub * kSubBytes;  // K (or V) stage
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kStages = (HD == 128) ? 3 : 6;
  static constexpr int kRingBytes = kStages * kStageBytes;  // 192 KB: one CTA per SM
  // K+V bytes of its chunk a CTA prefetches into L2 before the grid dependency wait:
  // 148 resident CTAs x 512 KB = 76 MB, within the 126 MB L2.
  static constexpr int kPrefetchBytes = 512 * 1024;
  static constexpr int kWarps = 8;                          // compute warps
  static constexpr int kThreads = (kWarps + 1) * 32;        // + one TMA producer warp
  // barriers (full[kStages], empty[kStages], combine) + flags after the ring
  static constexpr int kBarBytes = (2 * kStages + 1) * 8;
  static constexpr int kSmemBytes = kRingBytes + kBarBytes + 64 + 1024;
};

#define GQA_CBAR() asm volatile("bar.sync 1, %0;" ::"n"(CT) : "memory")  // the compute warps

// FP8: K and V are e4m3 (HD = 128, so a key row is 128 bytes, the shared-memory
// geometry of a 16-bit HD = 64 row); Q and O keep the 16-bit I/O type. Both MMAs
// then run in f16: Q is converted once, K and V fragments are converted exactly
// from e4m3 after ldmatrix, and P is packed as f16 (P <= 1).
//
// NT (at most 8 packed rows: decode): the MMAs run transposed, keys as M and the
// rows as N, so an m16n8k16 carries 16 keys x 8 rows instead of 8 keys x 16 rows
// of which at most 8 are real: S^T = K Q^T, then O^T += V^T P^T with P^T's
// fragments from movmatrix. Half the MMAs and half the exp2 work per key.
template <int HD, bool BF16, int RG, bool FP8 = false, bool NT = false>
__global__ void __launch_bounds__(288, 1)
    gqa_stream_kernel(const StreamParams p, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap) {
  static_assert(!FP8 || HD == 128, "fp8 K/V rows are 128 bytes");
  static_assert(!NT || RG == 1, "the transposed form is the one-row-group kernel");
  using Cfg = StreamCfg<FP8 ? 64 : HD>;  // ring geometry (bytes per key row)
  constexpr bool MMA_BF16 = BF16 && !FP8;  // operand type of both MMAs
  constexpr int NW = Cfg::kWarps;
  constexpr int KS = NW / RG;           // warps sharing one row group split the stage's keys
  constexpr int NKW = Cfg::kBN / KS;    // keys per warp per stage (16, 32, 64)
  constexpr int NNB = NKW / 8;          // n8 blocks per warp per stage
  constexpr int NDB = HD / 8;           // n8 blocks along d
  constexpr int NKS = HD / 16;          // k16 steps along d
  constexpr int CT = NW * 32;           // compute threads
  static_assert(NKW >= 16, "a warp needs at least one k16 block of keys");
  static_assert(!NT || NKW == 16, "transposed: one m16 block of keys per warp and stage");
  constexpr int NACC = NT ? HD / 16 : NDB;  // accumulator fragments

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* const smem = smem_raw + (base - raw_base);
  const uint32_t bar_full = base + Cfg::kRingBytes;
  const uint32_t bar_empty = bar_full + Cfg::kStages * 8;
  const uint32_t bar_comb = bar_empty + Cfg::kStages * 8;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kRingBytes + Cfg::kBarBytes);
  int* last_flag = reinterpret_cast<int*>(smem + Cfg::kRingBytes + Cfg::kBarBytes + 4);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  // ---- work item -----------------------------------------------------------
  const int split = blockIdx.x % p.nsplit;
  const int unit = blockIdx.x / p.nsplit;
  const int mt = unit % p.n_mtiles;
  const int kvh = (unit / p.n_mtiles) % p.hkv;
  const int b = unit / (p.n_mtiles * p.hkv);
  int off = p.seq_kv_total - p.seq_q;  // bottom-right causal offset (global; paged: per sequence)
  const bool paged = p.block_table != nullptr;

  // The producer thread initialises the barriers; every thread then waits for the
  // previous grid on the stream before its first global access (the sequence length
  // of a paged call included), and the producer issues the first ring of loads
  // before the CTA-wide barrier, so HBM requests start at once.
  if (tid == CT) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, NW);
    }
    mbar_init(bar_comb, 1);
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
  // Dense K/V: the chunk's key range follows from the parameters alone, so the
  // producer warp asks for the first kPrefetchBytes of it in L2 before the grid
  // dependency wait. Under programmatic dependent launch this CTA becomes resident
  // as soon as a CTA of the previous grid leaves its SM, so these reads overlap the
  // previous grid's tail (its cross-warp merge, publish and combine), when HBM would
  // otherwise idle. The prefetch is a hint (the loads after the wait still read
  // through L2), so it cannot return stale data even if the previous grid writes
  // K or V. Paged calls skip it: their block table may be written by that grid.
  if (!paged && warp == NW) {
    int kv_end0 = p.seq_kv;
    if (p.causal) kv_end0 = min(kv_end0, min((mt + 1) * p.block_m, p.seq_q) - 1 + off - p.kv_offset + 1);
    const int kb = split * p.chunk;
    const int ke = min(min(kb + p.chunk, kv_end0), kb + Cfg::kPrefetchBytes / (Cfg::kStageBytes / Cfg::kBN));
    const int nbox = (ke > kb) ? (ke - kb + Cfg::kBox - 1) / Cfg::kBox : 0;
    for (int i = lane; i < nbox * Cfg::kNSub; i += 32) {
      const int key = kb + (i / Cfg::kNSub) * Cfg::kBox, c0 = (i % Cfg::kNSub) * 64;
      tma_prefetch_l2_4d(&kmap, c0, key, kvh, b);
      tma_prefetch_l2_4d(&vmap, c0, key, kvh, b);
    }
  }
  pdl_wait();

  // Highest key (local, exclusive) any valid row of this unit may see.
  int kv_end = p.seq_kv;
  if (paged) {
    // A length above the host's bound is clipped to it (the plan covers seq_kv keys);
    // the checked build reports such a call.
    (void)GQA_CHECK(p.seq_lens[b] <= p.seq_kv, 906);
    kv_end = max(0, min(kv_end, p.seq_lens[b]));
    off = kv_end - p.seq_q;  // the sequence's queries are its last seq_q positions
  }
  if (p.causal) {
    const int last_pos = min((mt + 1) * p.block_m, p.seq_q) - 1;
    kv_end = min(kv_end, last_pos + off - p.kv_offset + 1);
  }
  const int k_begin = split * p.chunk;
  const int k_end = min(k_begin + p.chunk, kv_end);
  const int n_stages = (k_end > k_begin) ? (k_end - k_begin + Cfg::kBN - 1) / Cfg::kBN : 0;

  // A stage holds one or two 64-key boxes of K and of V (the chunk's last stage may
  // be half). Paged calls look up the physical block of each box; the producer loads
  // those indices before it waits for the stage's slot, so the lookup overlaps the wait.
  auto stage_blocks = [&](int t, int& pb0, int& pb1) {
    pb0 = pb1 = 0;
    if (!paged) return;
    const int key0 = k_begin + t * Cfg::kBN;
    const int* row_bt = p.block_table + (int64_t)b * p.bt_stride;
    pb0 = row_bt[key0 >> p.block_shift];
    if (key0 + Cfg::kBox < k_end) pb1 = row_bt[(key0 + Cfg::kBox) >> p.block_shift];
  };
  auto issue = [&](int t, int pb0, int pb1) {
    const int slot = t % Cfg::kStages;
    const uint32_t full = bar_full + 8 * slot;
    const int key0 = k_begin + t * Cfg::kBN;
    const int halves = (min(Cfg::kBN, k_end - key0) + Cfg::kBox - 1) / Cfg::kBox;
    mbar_arrive_expect_tx(full, halves * 2 * Cfg::kNSub * Cfg::kBoxBytes);
    const uint32_t kdst = base + slot * Cfg::kStageBytes;
    const uint32_t vdst = kdst + Cfg::kTileBytes;
    for (int h = 0; h < halves; ++h) {
      const int key = key0 + h * Cfg::kBox;
      // dense: (d, key, head, batch); paged: (d, head, position in block, physical block)
      const int c1 = paged ? kvh : key;
      const int c2 = paged ? (key & ((1 << p.block_shift) - 1)) : kvh;
      const int c3 = paged ? (h ? pb1 : pb0) : b;
#pragma unroll
      for (int s = 0; s < Cfg::kNSub; ++s) {
        const uint32_t o = s * Cfg::kSubBytes + h * Cfg::kBoxBytes;
        tma_load_4d(kdst + o, &kmap, full, s * 64, c1, c2, c3);
        tma_load_4d(vdst + o, &vmap, full, s * 64, c1, c2, c3);
      }
    }
  };
  const int n_first = min(n_stages, Cfg::kStages);
  if (tid == CT) {
    int pb[Cfg::kStages][2];
#pragma unroll
    for (int t = 0; t < Cfg::kStages; ++t)
      if (t < n_first) stage_blocks(t, pb[t][0], pb[t][1]);
#pragma unroll
    for (int t = 0; t < Cfg::kStages; ++t)
      if (t < n_first && !withheld_load(t)) issue(t, pb[t][0], pb[t][1]);
  }
  pdl_trigger();
  __syncthreads();

  if (warp == NW) {
    // ---------------------------------------------------------------- producer
    if (lane == 0 && n_stages > 0) {
      int t = n_first;
      for (; t < n_stages; ++t) {
        const int slot = t % Cfg::kStages;
        int pb0, pb1;
        stage_blocks(t, pb0, pb1);
        if (!mbar_wait(bar_empty + 8 * slot, (t / Cfg::kStages - 1) & 1, abort_flag, 101)) break;
        if (!withheld_load(t)) issue(t, pb0, pb1);
      }
      // On abort, let the loads already issued land before the CTA exits.
      if (t < n_stages) {
        for (int u = max(0, t - Cfg::kStages); u < t; ++u) {
          volatile int dummy = 0;
          if (!withheld_load(u)) mbar_wait(bar_full + 8 * (u % Cfg::kStages), (u / Cfg::kStages) & 1, &dummy, 102);
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------------- compute
  const int rg = warp % RG;
  const int ks = warp / RG;
  const int gr = lane >> 2;
  const int gc = lane & 3;

  // Packed rows owned by this thread: r0 = rg*16 + gr, r1 = r0 + 8 (NT: the softmax
  // rows 2gc, 2gc + 1, and Q row gr for the B fragments).
  int lim_r[2];  // local key limit (exclusive) for each row, clipped to the chunk
  const uint16_t* qrow[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    auto row_pos = [&](int r, int& g) {
      g = r / p.block_m;
      return mt * p.block_m + (r - g * p.block_m);
    };
    int g;
    const int rl = NT ? 2 * gc + h : rg * 16 + gr + 8 * h;
    const int pos_l = row_pos(rl, g);
    int lim = k_end;
    if (p.causal) lim = min(lim, pos_l + off - p.kv_offset + 1);
    lim_r[h] = lim;
    const int rq = NT ? gr : rl;
    const int pos = row_pos(rq, g);
    const bool valid = (rq < p.rows) && (pos < p.seq_q) && (!NT || h == 0);
    qrow[h] = valid ? p.q + b * p.q_sb + (int64_t)(kvh * p.group + g) * p.q_sh + (int64_t)pos * p.q_sm : nullptr;
  }

  // Q fragments (A operand, 16 rows x HD), loaded once.
  uint32_t qa[NKS][4];
  if constexpr (NT && FP8) {
    // B fragments of K Q^T: k16 step kk, row gr, d 16kk + 4gc..+3 (the e4m3 order).
#pragma unroll
    for (int kk = 0; kk < NKS; ++kk) {
      const uint2 q0 = qrow[0] ? *reinterpret_cast<const uint2*>(qrow[0] + kk * 16 + gc * 4) : make_uint2(0u, 0u);
      qa[kk][0] = to_f16x2<BF16>(q0.x);
      qa[kk][1] = to_f16x2<BF16>(q0.y);
      qa[kk][2] = qa[kk][3] = 0u;
    }
  } else if constexpr (NT) {
    // B fragments of K Q^T: k16 step kk, row gr, d 16kk + 2gc, +1 and 16kk + 2gc + 8, +9.
#pragma unroll
    for (int kk = 0; kk < NKS; ++kk) {
      const int d0 = kk * 16 + gc * 2;
      qa[kk][0] = qrow[0] ? *reinterpret_cast<const uint32_t*>(qrow[0] + d0) : 0u;
      qa[kk][1] = qrow[0] ? *reinterpret_cast<const uint32_t*>(qrow[0] + d0 + 8) : 0u;
      qa[kk][2] = qa[kk][3] = 0u;
    }
  } else if constexpr (FP8) {
    // k16 step kk covers d 16kk..16kk+15 in the order the e4m3 K fragments take
    // (k 2t, 2t+1 -> d 4t, 4t+1; k 2t+8, 2t+9 -> d 4t+2, 4t+3), in f16.
#pragma unroll
    for (int kk = 0; kk < NKS; ++kk) {
      const int d0 = kk * 16 + gc * 4;
      const uint2 z = make_uint2(0u, 0u);
      const uint2 q0 = qrow[0] ? *reinterpret_cast<const uint2*>(qrow[0] + d0) : z;
      const uint2 q1 = qrow[1] ? *reinterpret_cast<const uint2*>(qrow[1] + d0) : z;
      qa[kk][0] = to_f16x2<BF16>(q0.x);
      qa[kk][1] = to_f16x2<BF16>(q1.x);
      qa[kk][2] = to_f16x2<BF16>(q0.y);
      qa[kk][3] = to_f16x2<BF16>(q1.y);
    }
  } else {
#pragma unroll
    for (int kk = 0; kk < NKS; ++kk) {
      const int d0 = kk * 16 + gc * 2;
      qa[kk][0] = qrow[0] ? *reinterpret_cast<const uint32_t*>(qrow[0] + d0) : 0u;
      qa[kk][1] = qrow[1] ? *reinterpret_cast<const uint32_t*>(qrow[1] + d0) : 0u;
      qa[kk][2] = qrow[0] ? *reinterpret_cast<const uint32_t*>(qrow[0] + d0 + 8) : 0u;
      qa[kk][3] = qrow[1] ? *reinterpret_cast<const uint32_t*>(qrow[1] + d0 + 8) : 0u;
    }
  }

  float acc[NACC][4];
#pragma unroll
  for (int i = 0; i < NACC; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  const float scale = p.scale_log2;

  for (int t = 0; t < n_stages; ++t) {
    const int slot = t % Cfg::kStages;
    bool ok = mbar_wait(bar_full + 8 * slot, (t / Cfg::kStages) & 1, abort_flag, 103);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) break;
    const uint32_t kst = base + slot * Cfg::kStageBytes;
    const uint32_t vst = kst + Cfg::kTileBytes;
    const int key_w = k_begin + t * Cfg::kBN + ks * NKW;  // first key of this warp's block
    if (key_w < k_end && key_w + NKW > k_end) {
      // The block holding the chunk's end: keys past it are masked (P = 0), but a paged
      // sequence's last cache block holds stale slots there and 0 x NaN would still
      // reach O through the MMA, so this warp zeroes the V rows of those keys (only it
      // reads them). The stage is the chunk's last: no copy refills the slot afterwards.
      const int first = k_end - key_w;
      constexpr int kRowChunks = Cfg::kNSub * 8;  // 16-byte chunks of one V row
      for (int i = lane; i < (NKW - first) * kRowChunks; i += 32) {
        const int r = ks * NKW + first + i / kRowChunks, c = i % kRowChunks;
        const uint32_t addr = vst + (c >> 3) * Cfg::kSubBytes + r * 128 + (c & 7) * 16;
        asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0u) : "memory");
      }
      __syncwarp();
    }
    if constexpr (NT) {
      if (key_w < k_end) {
        // ---- S^T = K Q^T: 16 keys (M) x 8 rows (N). Two partial sums (even and odd
        // k16 steps) keep two MMA chains in flight. A 16-byte chunk of a key row is
        // one k16 step; ldmatrix gives lane (g, t) d 4t..4t+3 of keys g and g + 8.
        float st[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        const int krow = ks * NKW + (lane & 7) + ((lane >> 3) & 1) * 8;
        if constexpr (FP8) {
#pragma unroll
          for (int c = 0; c < HD / 16; c += 2) {
            uint32_t r[4];
            ldsm_x4(kst + sw128_off(krow, c + (lane >> 4)), r[0], r[1], r[2], r[3]);
#pragma unroll
            for (int h = 0; h < 2; ++h) {  // chunk c + h: keys 0-7 in r[2h], keys 8-15 in r[2h + 1]
              const uint32_t a[4] = {e4m3x2_to_f16x2(r[2 * h]), e4m3x2_to_f16x2(r[2 * h + 1]),
                                     e4m3x2_to_f16x2(r[2 * h] >> 16), e4m3x2_to_f16x2(r[2 * h + 1] >> 16)};
              mma_16816<false>(st[h], a, qa[c + h][0], qa[c + h][1]);
            }
          }
        } else {
          // k16 step kk = 16-byte chunks 2kk, 2kk + 1 of keys 0-7 and 8-15: the four
          // matrices of one ldmatrix are the A fragment as they land.
#pragma unroll
          for (int kk = 0; kk < NKS; ++kk) {
            const int chunk = 2 * kk + (lane >> 4);
            uint32_t a[4];
            ldsm_x4(kst + (chunk >> 3) * Cfg::kSubBytes + sw128_off(krow, chunk & 7), a[0], a[1], a[2], a[3]);
            mma_16816<MMA_BF16>(st[kk & 1], a, qa[kk][0], qa[kk][1]);
          }
        }
        // s[e]: key gr + 8 (e >> 1), row 2gc + (e & 1)
        float s[4], mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = key_w + gr + 8 * (e >> 1);
          const float x = (key < lim_r[e & 1]) ? (st[0][e] + st[1][e]) * scale : -INFINITY;
          s[e] = x;
          mx[e & 1] = fmaxf(mx[e & 1], x);
        }
        float alpha[2], mu[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // rows are spread over the lanes of one gc
          mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 4));
          mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 8));
          mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 16));
          const float m_new = fmaxf(m_run[h], mx[h]);
          mu[h] = (m_new == -INFINITY) ? 0.f : m_new;  // keeps fully-masked rows at p = 0, not NaN
          alpha[h] = fast_exp2(m_run[h] - mu[h]);
          m_run[h] = m_new;
        }
        float lsum[2] = {0.f, 0.f};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          s[e] = fast_exp2(s[e] - mu[e & 1]);
          lsum[e & 1] += s[e];
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) l_run[h] = l_run[h] * alpha[h] + lsum[h];
#pragma unroll
        for (int c = 0; c < NACC; ++c) {  // acc[c]: rows 2gc, 2gc + 1, 2gc, 2gc + 1
          acc[c][0] *= alpha[0];
          acc[c][1] *= alpha[1];
          acc[c][2] *= alpha[0];
          acc[c][3] *= alpha[1];
        }
        // ---- O^T += V^T P^T. P^T's B fragments: the 8 x 8 (key, row) blocks of P
        // transposed in registers. V^T's A fragments: transposed 8 x 16-byte loads of
        // keys 0-7 and 8-15; bytes (0, 2) are keys 2t, 2t + 1 at d = 2g (A row g),
        // bytes (1, 3) the same keys at d = 2g + 1 (A row g + 8).
        const uint32_t pb0 = movmatrix_t(pack2<MMA_BF16>(s[0], s[1]));  // keys 0-7
        const uint32_t pb1 = movmatrix_t(pack2<MMA_BF16>(s[2], s[3]));  // keys 8-15
        if constexpr (FP8) {
#pragma unroll
          for (int c = 0; c < HD / 16; c += 2) {
            uint32_t r[4];
            ldsm_x4_t(vst + sw128_off(krow, c + (lane >> 4)), r[0], r[1], r[2], r[3]);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint32_t lo = prmt(r[2 * h], 0u, 0x3120u);      // keys 0-7:  d even pair | d odd pair
              const uint32_t hi = prmt(r[2 * h + 1], 0u, 0x3120u);  // keys 8-15
              const uint32_t a[4] = {e4m3x2_to_f16x2(lo), e4m3x2_to_f16x2(lo >> 16), e4m3x2_to_f16x2(hi),
                                     e4m3x2_to_f16x2(hi >> 16)};
              mma_16816<false>(acc[c + h], a, pb0, pb1);
            }
          }
        } else {
          // d tile c (A rows = d 16c..16c+15): transposed loads of (keys 0-7, d lo),
          // (keys 0-7, d hi), (keys 8-15, d lo), (keys 8-15, d hi) are a0..a3.
          const int vrow = ks * NKW + (lane & 7) + (lane >> 4) * 8;
#pragma unroll
          for (int c = 0; c < NACC; ++c) {
            const int chunk = 2 * c + ((lane >> 3) & 1);
            uint32_t a[4];
            ldsm_x4_t(vst + (chunk >> 3) * Cfg::kSubBytes + sw128_off(vrow, chunk & 7), a[0], a[1], a[2], a[3]);
            mma_16816<MMA_BF16>(acc[c], a, pb0, pb1);
          }
        }
      }
    } else {
      if (key_w < k_end) {  // warp-uniform: blocks past the chunk end were not loaded
        // ---- S = Q K^T over this warp's NKW keys
        float s[NNB][4];
#pragma unroll
        for (int nb = 0; nb < NNB; ++nb) s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
        if constexpr (FP8) {
          // A 16-byte chunk of a key row is 16 e4m3 values of d, one k16 step: lane
          // (g, t) of an 8 x 16-byte ldmatrix gets d 4t..4t+3 of key g, i.e. both B
          // registers of the step in the order the Q fragments were loaded in.
#pragma unroll
          for (int kc = 0; kc < HD / 64; ++kc) {
#pragma unroll
            for (int nb = 0; nb < NNB; ++nb) {
              const int krow = ks * NKW + nb * 8 + (lane & 7);
              const int chunk = kc * 4 + (lane >> 3);
              uint32_t r[4];
              ldsm_x4(kst + sw128_off(krow, chunk), r[0], r[1], r[2], r[3]);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                mma_16816<false>(s[nb], qa[4 * kc + j], e4m3x2_to_f16x2(r[j]), e4m3x2_to_f16x2(r[j] >> 16));
            }
          }
        } else {
#pragma unroll
          for (int kc = 0; kc < HD / 32; ++kc) {
#pragma unroll
            for (int nb = 0; nb < NNB; ++nb) {
              const int krow = ks * NKW + nb * 8 + (lane & 7);
              const int chunk = kc * 4 + (lane >> 3);
              const uint32_t addr = kst + (chunk >> 3) * Cfg::kSubBytes + sw128_off(krow, chunk & 7);
              uint32_t b0, b1, b2, b3;
              ldsm_x4(addr, b0, b1, b2, b3);
              mma_16816<BF16>(s[nb], qa[2 * kc], b0, b1);
              mma_16816<BF16>(s[nb], qa[2 * kc + 1], b2, b3);
            }
          }
        }

        // ---- online softmax (log2 domain)
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int nb = 0; nb < NNB; ++nb) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int h = e >> 1;
            const int key = key_w + nb * 8 + gc * 2 + (e & 1);
            const float x = (key < lim_r[h]) ? s[nb][e] * scale : -INFINITY;
            s[nb][e] = x;
            mx[h] = fmaxf(mx[h], x);
          }
        }
        float alpha[2], mu[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
          mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
          const float m_new = fmaxf(m_run[h], mx[h]);
          mu[h] = (m_new == -INFINITY) ? 0.f : m_new;  // keeps fully-masked rows at p = 0, not NaN
          alpha[h] = fast_exp2(m_run[h] - mu[h]);
          m_run[h] = m_new;
        }
        float lsum[2] = {0.f, 0.f};
#pragma unroll
        for (int nb = 0; nb < NNB; ++nb) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float pv = fast_exp2(s[nb][e] - mu[e >> 1]);
            s[nb][e] = pv;
            lsum[e >> 1] += pv;
          }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) l_run[h] = l_run[h] * alpha[h] + lsum[h];
#pragma unroll
        for (int i = 0; i < NDB; ++i) {
          acc[i][0] *= alpha[0];
          acc[i][1] *= alpha[0];
          acc[i][2] *= alpha[1];
          acc[i][3] *= alpha[1];
        }

        // ---- O += P V
#pragma unroll
        for (int kk = 0; kk < NKW / 16; ++kk) {
          uint32_t pa[4];
          pa[0] = pack2<MMA_BF16>(s[2 * kk][0], s[2 * kk][1]);
          pa[1] = pack2<MMA_BF16>(s[2 * kk][2], s[2 * kk][3]);
          pa[2] = pack2<MMA_BF16>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
          pa[3] = pack2<MMA_BF16>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
          const int vrow = ks * NKW + kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          if constexpr (FP8) {
            // Transposed 8 x 16-byte loads of keys 0-7 and 8-15 of 16-d chunks c, c+1:
            // lane (g, t) gets keys 2t, 2t+1 x d 2g, 2g+1 of each. Bytes (0, 2) are the
            // B pair of column d = 2g, bytes (1, 3) that of d = 2g + 1, so chunk c
            // feeds accumulator blocks 2c (even d) and 2c + 1 (odd d).
#pragma unroll
            for (int c = 0; c < HD / 16; c += 2) {
              const int chunk = c + (lane >> 4);
              uint32_t r[4];
              ldsm_x4_t(vst + sw128_off(vrow, chunk), r[0], r[1], r[2], r[3]);
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const uint32_t lo = prmt(r[2 * h], 0u, 0x3120u);      // keys 0-7:  even pair | odd pair
                const uint32_t hi = prmt(r[2 * h + 1], 0u, 0x3120u);  // keys 8-15
                mma_16816<false>(acc[2 * (c + h)], pa, e4m3x2_to_f16x2(lo), e4m3x2_to_f16x2(hi));
                mma_16816<false>(acc[2 * (c + h) + 1], pa, e4m3x2_to_f16x2(lo >> 16), e4m3x2_to_f16x2(hi >> 16));
              }
            }
          } else {
#pragma unroll
            for (int dc = 0; dc < NDB; dc += 2) {
              const int chunk = dc + (lane >> 4);
              const uint32_t addr = vst + (chunk >> 3) * Cfg::kSubBytes + sw128_off(vrow, chunk & 7);
              uint32_t b0, b1, b2, b3;
              ldsm_x4_t(addr, b0, b1, b2, b3);
              mma_16816<BF16>(acc[dc], pa, b0, b1);
              mma_16816<BF16>(acc[dc + 1], pa, b2, b3);
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_empty + 8 * slot);
  }

  // Row sums are per-thread partials over the quad's columns (NT: over the lanes
  // of one gc, which hold the keys).
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if constexpr (NT) {
      l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 4);
      l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 8);
      l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 16);
    } else {
      l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
      l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
    }
  }

  // ---- merge the KS warps of each row group through shared memory
  GQA_CBAR();  // every compute warp is done with the ring
  // acc rows are padded to HD + 8 floats: the 8 row lanes of a float2 store then
  // start 8 banks apart and each store takes the minimum two wavefronts. Rows of
  // the upper half of a row group are stored only when the unit has them. The
  // transposed (decode) form stores scalars whose lanes span rows 2gc (gc = 0..3)
  // and 8 consecutive d: a pad of HD + 4 puts those rows 8 banks apart, so each
  // store is one wavefront (HD + 8 would put rows 0 and 4 on the same banks).
  constexpr int AS = NT ? HD + 4 : HD + 8;
  float* mbuf = reinterpret_cast<float*>(smem);  // [NW][16]
  float* lbuf = mbuf + NW * 16;                  // [NW][16]
  float* abuf = lbuf + NW * 16;                  // [NW][16][AS]
  static_assert((2 * NW * 16 + NW * 16 * AS) * 4 <= Cfg::kRingBytes, "merge buffers fit the ring");
  {
    float* aw = abuf + warp * 16 * AS;
    const bool upper = rg * 16 + 8 < p.rows;  // warp-uniform
    if constexpr (NT && FP8) {
      // acc[c]: d 16c + 2gr (+1 in [2], [3]) of rows 2gc ([0], [2]) and 2gc + 1.
      const float vs = p.v_scale;
#pragma unroll
      for (int c = 0; c < NACC; ++c) {
        const int d = c * 16 + gr * 2;
        *reinterpret_cast<float2*>(aw + (2 * gc) * AS + d) = make_float2(acc[c][0] * vs, acc[c][2] * vs);
        *reinterpret_cast<float2*>(aw + (2 * gc + 1) * AS + d) = make_float2(acc[c][1] * vs, acc[c][3] * vs);
      }
    } else if constexpr (NT) {
      // acc[c]: d 16c + gr ([0], [1]) and 16c + gr + 8 ([2], [3]) of rows 2gc, 2gc + 1.
#pragma unroll
      for (int c = 0; c < NACC; ++c) {
        const int d = c * 16 + gr;
        aw[(2 * gc) * AS + d] = acc[c][0];
        aw[(2 * gc + 1) * AS + d] = acc[c][1];
        aw[(2 * gc) * AS + d + 8] = acc[c][2];
        aw[(2 * gc + 1) * AS + d + 8] = acc[c][3];
      }
    } else if constexpr (FP8) {
      // Blocks 2c, 2c + 1 hold d = 16c + 4t + {0, 2} and {1, 3}: four consecutive d.
      const float vs = p.v_scale;
#pragma unroll
      for (int c = 0; c < HD / 16; ++c) {
        const int d = c * 16 + gc * 4;
        const float* e = acc[2 * c];
        const float* o = acc[2 * c + 1];
        *reinterpret_cast<float4*>(aw + gr * AS + d) = make_float4(e[0] * vs, o[0] * vs, e[1] * vs, o[1] * vs);
        if (upper)
          *reinterpret_cast<float4*>(aw + (gr + 8) * AS + d) =
              make_float4(e[2] * vs, o[2] * vs, e[3] * vs, o[3] * vs);
      }
    } else {
#pragma unroll
      for (int i = 0; i < NDB; ++i) {
        const int d = i * 8 + gc * 2;
        *reinterpret_cast<float2*>(aw + gr * AS + d) = make_float2(acc[i][0], acc[i][1]);
        if (upper) *reinterpret_cast<float2*>(aw + (gr + 8) * AS + d) = make_float2(acc[i][2], acc[i][3]);
      }
    }
    if constexpr (NT) {
      if (gr < 2) {  // rows 2gc, 2gc + 1 (gr 0); rows 8..15 do not exist (gr 1)
        const int r = 8 * gr + 2 * gc;
        mbuf[warp * 16 + r] = gr ? -INFINITY : m_run[0];
        mbuf[warp * 16 + r + 1] = gr ? -INFINITY : m_run[1];
        lbuf[warp * 16 + r] = gr ? 0.f : l_run[0];
        lbuf[warp * 16 + r + 1] = gr ? 0.f : l_run[1];
      }
    } else if (gc == 0) {
      mbuf[warp * 16 + gr] = m_run[0];
      mbuf[warp * 16 + gr + 8] = m_run[1];
      lbuf[warp * 16 + gr] = l_run[0];
      lbuf[warp * 16 + gr + 8] = l_run[1];
    }
  }
  GQA_CBAR();

  // This CTA's combined (M, L) of packed row r and its acc over columns d..d+3,
  // from the KS warps' partials of the row. Every thread that writes a row computes
  // the row's weights itself (KS loads and exp2s, the same values in the same order
  // for all of them): no barrier and no separate weights phase between the stores
  // above and the writes below.
  struct RowMerge {
    float M, L;
    float4 a;
  };
  auto merge_row = [&](int r, int d) {
    const int g_rg = r / 16, rr = r % 16;
    float mk[KS];
    float M = -INFINITY;
#pragma unroll
    for (int k2 = 0; k2 < KS; ++k2) {
      mk[k2] = mbuf[(k2 * RG + g_rg) * 16 + rr];
      M = fmaxf(M, mk[k2]);
    }
    const float Mu = (M == -INFINITY) ? 0.f : M;
    RowMerge out{M, 0.f, make_float4(0.f, 0.f, 0.f, 0.f)};
#pragma unroll
    for (int k2 = 0; k2 < KS; ++k2) {
      const int w = k2 * RG + g_rg;
      const float wt = fast_exp2(mk[k2] - Mu);
      out.L += wt * lbuf[w * 16 + rr];
      const float4 v = *reinterpret_cast<const float4*>(abuf + (w * 16 + rr) * AS + d);
      out.a.x += wt * v.x;
      out.a.y += wt * v.y;
      out.a.z += wt * v.z;
      out.a.w += wt * v.w;
    }
    return out;
  };

  const int n_rows = min(p.rows, RG * 16);
  constexpr int per_row = HD / 4;
  if (p.mode == kStreamOut) {
    for (int idx = tid; idx < n_rows * per_row; idx += CT) {
      const int r = idx / per_row, d = (idx - r * per_row) * 4;
      const int g = r / p.block_m, m = r - g * p.block_m, pos = mt * p.block_m + m;
      if (pos >= p.seq_q) continue;
      const RowMerge mr = merge_row(r, d);
      const float4 a = mr.a;
      const float inv = 1.f / mr.L;  // l == 0 (no visible key) -> NaN, as the reference
      uint2 pk;
      pk.x = pack2<BF16>(a.x * inv, a.y * inv);
      pk.y = pack2<BF16>(a.z * inv, a.w * inv);
      uint16_t* dst = reinterpret_cast<uint16_t*>(p.o) + b * p.o_sb + (int64_t)(kvh * p.group + g) * p.o_sh +
                      (int64_t)pos * p.o_sm + d;
      *reinterpret_cast<uint2*>(dst) = pk;
    }
    return;
  }
  if (p.mode == kStreamRefPartial) {
    for (int idx = tid; idx < n_rows * per_row; idx += CT) {
      const int r = idx / per_row, d = (idx - r * per_row) * 4;
      const int g = r / p.block_m, m = r - g * p.block_m, pos = mt * p.block_m + m;
      if (pos >= p.seq_q) continue;
      const int head = kvh * p.group + g;
      const RowMerge mr = merge_row(r, d);
      const float4 a = mr.a;
      float* ap = p.acc_p + b * p.a_sb + head * p.a_sh + (int64_t)pos * p.a_sm + (int64_t)split * p.a_ss;
      ap[(int64_t)(d + 0) * p.a_sd] = a.x;
      ap[(int64_t)(d + 1) * p.a_sd] = a.y;
      ap[(int64_t)(d + 2) * p.a_sd] = a.z;
      ap[(int64_t)(d + 3) * p.a_sd] = a.w;
      if (d == 0) {
        const int64_t po = b * p.p_sb + head * p.p_sh + (int64_t)pos * p.p_sm + (int64_t)split * p.p_ss;
        p.m_p[po] = mr.M;
        p.l_p[po] = mr.L;
      }
    }
    return;
  }

  // ---- kStreamFused / kStreamFusedPartial: publish this chunk's partial.
  const int64_t wbase = ((int64_t)unit * p.nsplit + split) * p.rows;
  for (int idx = tid; idx < n_rows * per_row; idx += CT) {
    const int r = idx / per_row, d = (idx - r * per_row) * 4;
    const RowMerge mr = merge_row(r, d);
    __stcg(reinterpret_cast<float4*>(p.ws_acc + (wbase + r) * HD + d), mr.a);
    if (d == 0) {
      __stcg(p.ws_m + wbase + r, mr.M);
      __stcg(p.ws_l + wbase + r, mr.L);
    }
  }
  // The CTA barrier orders every thread's partial stores before thread 0's
  // release-acquire ticket (fences are cumulative); the last CTA acquires them.
  GQA_CBAR();
  if (tid == 0) {
    unsigned ticket;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(ticket) : "l"(p.ws_cnt + unit) : "memory");
    *last_flag = (ticket == (unsigned)(p.nsplit - 1)) ? 1 : 0;
  }
  GQA_CBAR();
  if (!*last_flag) return;

  // ---- last CTA of the unit: log-sum-exp combine of all chunk partials.
  // Shared-memory layout (the ring is free now):
  //   sm_m, sm_l [nsplit][rows]        partial m and l
  //   cacc [nsplit][rows][HD]          the unit's acc partials, staged by one bulk copy when they fit
  const int64_t ubase = (int64_t)unit * p.nsplit * p.rows;
  const int nsr = p.nsplit * n_rows;
  float* sm_m = reinterpret_cast<float*>(smem);
  float* sm_l = sm_m + nsr;
  const uint32_t small_bytes = ((uint32_t)(2 * nsr) * 4u + 15u) & ~15u;
  const uint32_t acc_bytes = (uint32_t)nsr * HD * 4u;
  const bool staged = small_bytes + acc_bytes <= (uint32_t)Cfg::kRingBytes;
  float* cacc = reinterpret_cast<float*>(smem + small_bytes);
  if (staged && tid == 0) {
    // Other CTAs wrote the partials with generic stores; this read goes through the async proxy.
    asm volatile("fence.proxy.async.global;" ::: "memory");
    mbar_arrive_expect_tx(bar_comb, acc_bytes);
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(cacc)),
                 "l"(reinterpret_cast<uint64_t>(p.ws_acc + ubase * HD)), "r"(acc_bytes), "r"(bar_comb)
                 : "memory");
  }
  for (int i = tid; i < nsr; i += CT) {
    sm_m[i] = __ldcg(p.ws_m + ubase + i);
    sm_l[i] = __ldcg(p.ws_l + ubase + i);
  }
  GQA_CBAR();
  if (staged) {
    // Waited for even after an abort: the bulk copy must land before the CTA exits.
    volatile int no_abort = 0;
    mbar_wait(bar_comb, 0, &no_abort, 104);
  }
  for (int idx = tid; idx < n_rows * per_row; idx += CT) {
    const int r = idx / per_row, d = (idx - r * per_row) * 4;
    const int g = r / p.block_m, m = r - g * p.block_m, pos = mt * p.block_m + m;
    if (pos >= p.seq_q) continue;
    // The row's weights over the unit's chunks, w_s = exp2(m_s - max_s m_s), and its
    // L = sum_s w_s l_s, computed by every thread that writes the row (the same values
    // in the same order), so no separate weights phase and barrier precede the sum.
    float M = -INFINITY;
    for (int s2 = 0; s2 < p.nsplit; ++s2) M = fmaxf(M, sm_m[s2 * n_rows + r]);
    const float Mu = (M == -INFINITY) ? 0.f : M;
    float L = 0.f;
    // Splits in batches of kCombBatch: every load of a batch is issued before the
    // first FMA, so a batch costs one load latency instead of one per split. The
    // sum runs in split order, as the reference's reduce does.
    constexpr int kCombBatch = 8;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    auto accumulate = [&](auto load) {
      for (int s0 = 0; s0 < p.nsplit; s0 += kCombBatch) {
        float wt[kCombBatch];
        float4 v[kCombBatch];
#pragma unroll
        for (int u = 0; u < kCombBatch; ++u) {
          if (s0 + u < p.nsplit) {
            wt[u] = fast_exp2(sm_m[(s0 + u) * n_rows + r] - Mu);
            v[u] = load(s0 + u);
          }
        }
#pragma unroll
        for (int u = 0; u < kCombBatch; ++u) {
          if (s0 + u < p.nsplit) {
            L += wt[u] * sm_l[(s0 + u) * n_rows + r];
            a.x += wt[u] * v[u].x;
            a.y += wt[u] * v[u].y;
            a.z += wt[u] * v[u].z;
            a.w += wt[u] * v[u].w;
          }
        }
      }
    };
    if (staged) {
      accumulate([&](int s2) { return *reinterpret_cast<const float4*>(cacc + (s2 * n_rows + r) * HD + d); });
    } else {
      accumulate([&](int s2) {
        return __ldcg(reinterpret_cast<const float4*>(p.ws_acc + (ubase + (int64_t)s2 * p.rows + r) * HD + d));
      });
    }
    const int head = kvh * p.group + g;
    if (p.mode == kStreamFused) {
      const float inv = 1.f / L;  // L == 0 (no visible key) -> NaN, as the reference
      uint2 pk;
      pk.x = pack2<BF16>(a.x * inv, a.y * inv);
      pk.y = pack2<BF16>(a.z * inv, a.w * inv);
      uint16_t* dst =
          reinterpret_cast<uint16_t*>(p.o) + b * p.o_sb + (int64_t)head * p.o_sh + (int64_t)pos * p.o_sm + d;
      *reinterpret_cast<uint2*>(dst) = pk;
    } else if (p.npeer > 0) {
      const int64_t ro = ((int64_t)b * p.hq + head) * p.seq_q + pos;
      const int64_t off = (int64_t)(*p.epoch & 1ull) * p.peer_parity + (int64_t)p.my_rank * p.peer_slot;
      for (int i = 0; i < p.npeer; ++i) {
        float* dst = p.peer_base[i] + off;
        *reinterpret_cast<float4*>(dst + p.pk_acc + ro * HD + d) = a;
        if (d == 0) {
          dst[ro] = M;
          dst[p.pk_rows + ro] = L;
        }
      }
    } else {
      const int64_t ro = ((int64_t)b * p.hq + head) * p.seq_q + pos;
      *reinterpret_cast<float4*>(p.acc_out + ro * HD + d) = a;
      if (d == 0) {
        p.m_out[ro] = M;
        p.l_out[ro] = L;
      }
    }
  }
  if (p.mode == kStreamFusedPartial && p.npeer > 0) {
    // Every compute thread's peer stores precede thread 0's releases (the barrier
    // orders them, the release is cumulative): a rank whose counter for this source
    // has grown sees this unit's rows.
    GQA_CBAR();
    if (tid == 0) {
      for (int i = 0; i < p.npeer; ++i)
        asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(p.peer_cnt[i] + p.my_rank) : "memory");
    }
  }
  if (tid == 0) p.ws_cnt[unit] = 0u;  // ready for the next call on this workspace
}

#undef GQA_CBAR

}  // namespace gqa
