// K2: flash attention on the 5th-generation tensor cores (tcgen05), S and P in TMEM.
//
// Computes, for every (sequence, head), softmax(q k^T * hd^-0.5 + mask) v over the
// packed valid-token layout -- the score/mask/softmax/PV sequence of the reference's
// BaselineSelfAttention.forward (benchmarks/torch_transformer_benchmark.py:97-117):
// causal triu(1) mask (:99-103), key-padding mask (:105-108), fp32 softmax (:111),
// probs @ v (:112).  Packing keeps token order inside a sequence, so the key-padding
// mask is "key < valid length" and the causal mask compares packed positions.
//
// Work item = one (sequence, head, NT x 128 query rows) = NT 128-row query tiles (NT = 2,
// or 1 at head_dim 256); the two sides swap query tiles on alternate items.  The CTA is persistent over the longest-first work list and runs
// 11 warps:
//   warp 8      TMA: Q tiles (double-buffered across items), K/V tiles (STAGES ring)
//   warps 9/10  issue tcgen05.mma for query tile 0 / 1 (the whole warp runs the loop,
//               one elected lane issues): S_t = Q_t K_j^T (M=128, N=128, K=hd) into
//               TMEM, and O_t += P_t V_j with P_t read from TMEM (A operand)
//   warps 0-3   softmax for query tile 0 (one thread = one query row = one TMEM lane)
//   warps 4-7   softmax for query tile 1
// P has its own TMEM buffer, so S_t(j+1) is issued as soon as the softmax threads have
// read S_t(j) into registers (s_free): the tensor core computes the next scores while
// the softmax works on the current ones, and neither warpgroup waits for an MMA in the
// steady state -- the exponentials (MUFU) set the pace.  A softmax thread loads its 128
// scores, releases the S buffer, applies the masks, updates the running max (rescaling
// O in TMEM only when the max grows by more than 2^8, lazily), waits until the previous
// P V has read the P buffer (pv_done), writes P as packed fp16 and signals the MMA warp
// (p_full).  At the end of an item it normalises O by the row sum and stores the rows.
//
// TMEM (512 columns), head_dim <= 64: S0 [0,128) S1 [128,256) P0 [256,320)
// P1 [320,384) O0 [384,384+hd) O1 [448,448+hd).
//
// head_dim 128 / 256: the O accumulators take 256 columns, so P has no buffer of its
// own: the softmax writes P_t over the first 64 columns of S_t, and the MMA warp issues
// the next S_t into that buffer only after P_t V has completed (it waits on pv_done; the
// tcgen05 ordering rules do not order two MMAs with different accumulators).  Then
// s_full also tells the softmax that the previous P V is done, so it needs neither
// s_free nor pv_done.  head_dim 128: S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512).
// head_dim 256 (NT = 1): S0 [0,128) O0 [256,512).  Q/K/V tiles of head_dim >= 64 are
// moved as head_dim/64 boxes of 64 columns (one 128-byte swizzle atom wide each).
//
// Every wait is bounded (TTTJ wait limit); on a timeout the role records
// TTTJ_DEV_TIMEOUT_ATTN in the status word, raises the CTA abort flag and unwinds.
//
// Sequence isolation: the K/V tile holding a sequence's last keys also holds rows of
// the next sequence of the packed layout (or rows no forward of this shape wrote
// since), which may be NaN or Inf.  Their scores are replaced by -inf (P = 0), and
// before the first P V of such a tile the MMA warp zeroes its V rows past the sequence
// end in shared memory, since 0 * NaN would still reach the output.  Query rows past
// the end (the next sequence's) never decide whether a warp rescales O, so a
// sequence's output does not depend on any other sequence's values.
#pragma once
#include "common.cuh"
#include "params.h"

namespace tttj {

// QB: Q buffers (work items in flight) at head_dim <= 64.  Two, with four K/V stages
// at head_dim 64, suit sequences of at most 256 tokens (items of one or two key tiles:
// the deeper ring keeps the next items' tiles coming); three, with three K/V stages (the
// shared memory holds no more), suit sequences of up to 2048 (measured: C5 attention 156
// vs 166 us, C2 26.7 vs 26.2 us; C4's 8192-token sequences no better).  The launcher
// picks by the longest sequence the plan allows.
template <int HD, int QB = 2>
struct AtcSmem {
  static_assert(HD == 32 || HD == 64 || HD == 128 || HD == 256, "head_dim layout");
  static constexpr int NT = HD == 256 ? 1 : 2;   // query tiles per work item
  static constexpr bool P_ALIAS = HD >= 128;     // P written over its S buffer
  static constexpr int QBUF = HD >= 128 ? 1 : QB;  // Q buffers (items in flight)
  static constexpr int QS = QBUF < 2 ? 2 : QBUF;  // Q barrier / info slots
  static constexpr int STAGES = HD == 32 ? 4 : HD == 64 ? (QB > 2 ? 3 : 4) : HD == 128 ? 2 : 1;
  static constexpr int BOX_COLS = HD < 64 ? HD : 64;  // TMA box width (one swizzle atom)
  static constexpr int NBOX = HD / BOX_COLS;
  static constexpr int BOX_BYTES = ATC_BM * BOX_COLS * 2;
  static constexpr int Q_TILE = ATC_BM * HD * 2;
  static constexpr int KV_TILE = ATC_BN * HD * 2;
  static constexpr int Q_BYTES = QBUF * NT * Q_TILE;
  static constexpr int KV_BYTES = STAGES * 2 * KV_TILE;
  static constexpr int NBAR = QS + QS + 2 * STAGES + 2 + 2 + 2 + 2 + 2 + 2 + 2;
  static constexpr int INFO_BYTES = QS * 64;  // decoded item (AtcItem, 40 B) per Q buffer
  // Epilogue staging per softmax warp: its 32 output rows x HD fp16 (head_dim <= 64;
  // wider heads store straight from registers).
  static constexpr bool STAGED_EPI = HD <= 64;
  static constexpr int EPI_ROW = HD * 2;
  static constexpr int EPI_BYTES = STAGED_EPI ? 8 * 32 * EPI_ROW : 0;
  static constexpr int TOTAL = Q_BYTES + KV_BYTES + NBAR * 8 + 16 + INFO_BYTES + EPI_BYTES + 1024;
  static constexpr uint32_t TMEM_S0 = 0, TMEM_S1 = 128;
  static constexpr uint32_t TMEM_P0 = P_ALIAS ? TMEM_S0 : 256, TMEM_P1 = P_ALIAS ? TMEM_S1 : 320;
  static constexpr uint32_t TMEM_O0 = HD <= 64 ? 384 : 256, TMEM_O1 = HD <= 64 ? 448 : 384;
};

struct AtcItem {
  int b, h, seq0, len, q0;
  int n[2];   // KV tiles streamed by query tile 0 / 1 (0 = tile empty)
  int kv_end[2];
  int n_kv;   // KV tiles loaded for the item; -1 marks "no more items"
};
static_assert(sizeof(AtcItem) <= 64, "item info slot is 64 bytes");

template <bool CAUSAL, int NT>
__device__ __forceinline__ AtcItem atc_decode(const AtcParams& p, int it) {
  AtcItem w;
  const int2 e = p.items[it];
  w.b = e.x;
  w.h = e.y & 0xff;
  w.q0 = (e.y >> 8) * (NT * ATC_BM);
  w.seq0 = p.seq_off[w.b];
  w.len = p.seq_off[w.b + 1] - w.seq0;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int r0 = w.q0 + t * ATC_BM;
    const int end = CAUSAL ? min(w.len, r0 + ATC_BM) : w.len;
    w.kv_end[t] = end;
    w.n[t] = (t < NT && r0 < w.len) ? (end + ATC_BN - 1) / ATC_BN : 0;
  }
  w.n_kv = max(w.n[0], w.n[1]);
  return w;
}

// K-major descriptor of head-dim step kk (16 elements) of a Q or K tile stored as
// NBOX boxes of [128 rows][BOX_COLS].
template <int HD>
__device__ __forceinline__ uint64_t atc_desc_qk(uint32_t tile, int kk) {
  if constexpr (HD == 32) {
    return desc_kmajor_sw64(tile) + (uint64_t)(2 * kk);
  } else {
    return desc_kmajor_sw128(tile + (uint32_t)((kk >> 2) * AtcSmem<HD>::BOX_BYTES)) +
           (uint64_t)(2 * (kk & 3));
  }
}
// Which query tile of the CTA's k-th item side t (a softmax warpgroup with its MMA warp
// and TMEM buffers) handles.  Causal items are uneven -- the upper query tile streams
// one key tile more than the lower one, and for sequences of <= 256 tokens that is
// twice the work -- so the sides swap tiles on alternate items and share the long ones
// (measured: C5 attention about 5% fewer cycles, C2 / C3 unchanged).
template <int NT>
__device__ __forceinline__ int atc_query_tile(int t, int k) {
  return NT == 2 ? (t ^ (k & 1)) : t;
}

template <int HD>
__device__ __forceinline__ uint64_t atc_desc_v(uint32_t addr) {
  // V tile [128 keys][HD] is the B operand (K = keys, N = HD) stored N-contiguous; the
  // 64-column boxes are the N atoms (LBO = box bytes), 8-key groups 1024 B apart.
  return HD == 32 ? desc_mnmajor_sw64(addr, AtcSmem<HD>::KV_TILE, 512)
                  : desc_mnmajor_sw128(addr, AtcSmem<HD>::BOX_BYTES, 1024);
}

#ifndef ATC_P_EARLY
#define ATC_P_EARLY 2
#endif

template <int HD, bool CAUSAL, int QB>
__global__ void __launch_bounds__(ATC_THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, const AtcParams p) {
  using SM = AtcSmem<HD, QB>;
  constexpr int STAGES = SM::STAGES;
  constexpr int NT = SM::NT;
  constexpr int QBUF = SM::QBUF;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sKV = sQ + SM::Q_BYTES;
  const uint32_t bar0 = sKV + SM::KV_BYTES;
  const uint32_t bar_q_full = bar0;                     // [QS]
  const uint32_t bar_q_empty = bar0 + 8 * SM::QS;       // [QS]
  const uint32_t bar_kv_full = bar0 + 16 * SM::QS;      // [STAGES]
  const uint32_t bar_kv_empty = bar_kv_full + 8 * STAGES;  // [STAGES]
  const uint32_t bar_s_full = bar_kv_empty + 8 * STAGES;   // [2]
  const uint32_t bar_p_full = bar_s_full + 16;             // [2]
  const uint32_t bar_o_full = bar_p_full + 16;             // [2]
  const uint32_t bar_o_free = bar_o_full + 16;             // [2]
  const uint32_t bar_s_free = bar_o_free + 16;             // [2] scores read by softmax
  const uint32_t bar_pv_done = bar_s_free + 16;            // [2] P V complete
  const uint32_t bar_drain = bar_pv_done + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + SM::Q_BYTES + SM::KV_BYTES + SM::NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // Decoded work item per Q buffer, written by the loader before it arms q_full, read
  // by the MMA and softmax warps after they waited on q_full (one global decode per item).
  AtcItem* info = reinterpret_cast<AtcItem*>(smem + SM::Q_BYTES + SM::KV_BYTES + SM::NBAR * 8 + 16);
  const uint32_t sEpi = smem_u32(smem + SM::Q_BYTES + SM::KV_BYTES + SM::NBAR * 8 + 16 + SM::INFO_BYTES);

  const int warp = warp_id();
  const int lane = lane_id();
  const uint64_t limit = p.wait_limit_ns;
  const int W = p.qkv_width;  // q | k | v column blocks of the qkv rows; ctx row stride

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmQKV);
    for (int i = 0; i < SM::QS; ++i) {
      mbar_init(bar_q_full + 8 * i, 1);
      // Released by the MMA warp's commit after the item's last Q K^T and by every
      // softmax thread once it copied the item's decoded info out of the slot.
      mbar_init(bar_q_empty + 8 * i, NT + NT * ATC_BM);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_s_full + 8 * i, 1);
      mbar_init(bar_p_full + 8 * i, ATC_BM);
      mbar_init(bar_o_full + 8 * i, 1);
      mbar_init(bar_o_free + 8 * i, ATC_BM);
      mbar_init(bar_s_free + 8 * i, ATC_BM);
      mbar_init(bar_pv_done + 8 * i, 1);
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_kv_full + 8 * s, 1);
      mbar_init(bar_kv_empty + 8 * s, NT);  // one arrival per MMA warp
    }
    mbar_init(bar_drain, 1);
    mbar_init(bar_drain + 8, 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  griddep_wait();
  griddep_launch();
  const int n_items = *p.item_count;

  if (warp == 8) {
    // ------------------------------------------------------------ TMA loader
    if (lane == 0) {
      bool ok = true;
      long kvc = 0;  // KV tiles issued
      int k = 0;     // items issued (including the final "no more items" marker)
      for (;; ++k) {
        // Dynamic scheduling: the next item of the longest-first list goes to the
        // first CTA that asks for it.
        const int it = atomicAdd(p.work_counter, 1);
        const bool stop = it >= n_items;
        AtcItem w;
        if (!stop) {
          w = atc_decode<CAUSAL, NT>(p, it);
        } else {
          w.n_kv = -1;
          w.n[0] = w.n[1] = 0;
        }
        const int qb = k % QBUF;
        if (!mbar_wait(bar_q_empty + 8 * qb, ((k / QBUF) & 1) ^ 1u, abort_flag, limit)) {
          ok = false;
          break;
        }
        info[qb] = w;  // published by the release of the arrive below
        if (stop) {
          mbar_arrive(bar_q_full + 8 * qb);
          break;
        }
        const int nq = w.n[1] > 0 ? 2 : 1;
        mbar_arrive_expect_tx(bar_q_full + 8 * qb, nq * SM::Q_TILE);
        for (int t = 0; t < nq; ++t)
          for (int x = 0; x < SM::NBOX; ++x)
            tma_load_2d(sQ + (qb * NT + t) * SM::Q_TILE + x * SM::BOX_BYTES, &tmQKV,
                        bar_q_full + 8 * qb, w.h * HD + x * SM::BOX_COLS, w.seq0 + w.q0 + t * ATC_BM);
        for (int j = 0; j < w.n_kv; ++j, ++kvc) {
          const int st = (int)(kvc % STAGES);
          if (!mbar_wait(bar_kv_empty + 8 * st, (uint32_t)((kvc / STAGES) & 1) ^ 1u, abort_flag,
                         limit)) {
            ok = false;
            break;
          }
          const uint32_t dst = sKV + st * 2 * SM::KV_TILE;
          mbar_arrive_expect_tx(bar_kv_full + 8 * st, 2 * SM::KV_TILE);
          for (int x = 0; x < SM::NBOX; ++x) {
            tma_load_2d(dst + x * SM::BOX_BYTES, &tmQKV, bar_kv_full + 8 * st,
                        W + w.h * HD + x * SM::BOX_COLS, w.seq0 + j * ATC_BN);
            tma_load_2d(dst + SM::KV_TILE + x * SM::BOX_BYTES, &tmQKV, bar_kv_full + 8 * st,
                        2 * W + w.h * HD + x * SM::BOX_COLS, w.seq0 + j * ATC_BN);
          }
        }
        if (!ok) break;
      }
      if (!ok) {
        *abort_flag = 1;
        report_status(p.status, TTTJ_DEV_TIMEOUT_ATTN);
        // Let issued loads land before the CTA can exit.
        for (long j = kvc > STAGES ? kvc - STAGES : 0; j < kvc; ++j)
          mbar_wait(bar_kv_full + 8 * (int)(j % STAGES), (uint32_t)((j / STAGES) & 1), nullptr,
                    limit);
        for (int i = k > QBUF ? k - QBUF : 0; i < k; ++i)
          mbar_wait(bar_q_full + 8 * (i % QBUF), (uint32_t)((i / QBUF) & 1), nullptr, limit);
      }
    }
  } else if (warp == 9 || (warp == 10 && NT == 2)) {
    // ------------------------------------------------------------ MMA issuers
    // One issuing warp per query tile, each following only its own tile's events, so
    // neither tile's MMAs wait for the other tile's softmax (a single issuer serving
    // both in a fixed order keeps the two softmax warpgroups in lockstep).  The whole
    // warp runs the loop (barrier results combined with a vote, item fields broadcast
    // from lane 0, so descriptors stay warp-uniform); one elected lane issues each
    // tcgen05.mma / commit.  A K/V stage is released by both warps (two arrivals); a
    // K/V tile a query tile does not use is released after it landed, which keeps the
    // releases in stage order.
    constexpr unsigned FULL = 0xffffffffu;
    const int t = warp - 9;
    {
      constexpr uint32_t idesc_s = idesc_f16_f32(ATC_BM, ATC_BN);
      constexpr uint32_t idesc_o = idesc_f16_f32(ATC_BM, HD, 0, 1);
      // 16 keys of V: 16 rows of the box (64 B rows at head_dim 32, 128 B otherwise).
      constexpr uint32_t v_step = HD == 32 ? (1024u >> 4) : (2048u >> 4);
      const uint32_t s_col = t == 0 ? SM::TMEM_S0 : SM::TMEM_S1;
      const uint32_t p_col = t == 0 ? SM::TMEM_P0 : SM::TMEM_P1;
      const uint32_t o_col = t == 0 ? SM::TMEM_O0 : SM::TMEM_O1;
      bool ok = true;
      bool issued = false;
      long kvc = 0;        // KV tiles of all items so far (global count)
      long kv_waited = -1;  // highest KV tile index whose arrival this warp observed
      long pc = 0, sfc = 0, oc = 0, pvc = 0;  // p_full / s_free / o_free / pv_done waits
      int k = 0;
      auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
        if (!__all_sync(FULL, mbar_wait(bar, parity, abort_flag, limit))) {
          ok = false;
          return false;
        }
        tc_fence_after();
        return true;
      };
      auto ensure_kv = [&](long idx) -> bool {
        while (kv_waited < idx) {
          ++kv_waited;
          if (!wait(bar_kv_full + 8 * (int)(kv_waited % STAGES), (uint32_t)((kv_waited / STAGES) & 1)))
            return false;
        }
        return true;
      };
      for (; ok; ++k) {
        const int qb = k % QBUF;
        if (!wait(bar_q_full + 8 * qb, (k / QBUF) & 1)) break;
        const int n_kv = __shfl_sync(FULL, info[qb].n_kv, 0);
        if (n_kv < 0) break;  // no more items
        // Query tile of this item handled by this warp's side (see atc_query_tile).
        const int tq = atc_query_tile<NT>(t, k);
        const int n = __shfl_sync(FULL, info[qb].n[tq], 0);
        const uint32_t qaddr = sQ + (qb * NT + tq) * SM::Q_TILE;
        auto issue_s = [&](long kv_idx) {
          const uint32_t kaddr = sKV + (int)(kv_idx % STAGES) * 2 * SM::KV_TILE;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            mma_f16_ss_warp(tmem + s_col, atc_desc_qk<HD>(qaddr, kk), atc_desc_qk<HD>(kaddr, kk),
                            idesc_s, kk > 0 ? 1u : 0u);
          mma_commit_warp(bar_s_full + 8 * t);
          issued = true;
        };
        // V rows of the tile at item key tile j_rel past the sequence end: zeroed in
        // shared memory (every 16-byte chunk of a row stays in that row under the
        // swizzle) and made visible to the tensor core before any P V reads them.  Both
        // MMA warps may do it for the same tile; they write the same zeros.
        const int seq_len = __shfl_sync(FULL, info[qb].len, 0);
        auto clean_v = [&](long kv_idx, int j_rel) {
          const int keep = seq_len - j_rel * ATC_BN;  // rows of this sequence (>= 1)
          if (keep >= ATC_BN) return;                 // warp-uniform
          constexpr int ROW_BYTES = SM::BOX_COLS * 2;
          constexpr int CH = ROW_BYTES / 16;
          const uint32_t vaddr = sKV + (int)(kv_idx % STAGES) * 2 * SM::KV_TILE + SM::KV_TILE;
          const int n16 = (ATC_BN - keep) * CH;
#pragma unroll 1
          for (int x = 0; x < SM::NBOX; ++x)
            for (int i = lane; i < n16; i += 32) {
              const uint32_t a = vaddr + (uint32_t)(x * SM::BOX_BYTES + (keep + i / CH) * ROW_BYTES +
                                                    (i % CH) * 16);
              asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0u) : "memory");
            }
          fence_proxy_async_smem();
          __syncwarp();
        };
        auto issue_pv = [&](long kv_idx, bool accumulate) {
          const uint32_t vaddr = sKV + (int)(kv_idx % STAGES) * 2 * SM::KV_TILE + SM::KV_TILE;
          const uint64_t vd = atc_desc_v<HD>(vaddr);
#pragma unroll
          for (int kk = 0; kk < ATC_BN / 16; ++kk)
            mma_f16_ts_warp(tmem + o_col, tmem + p_col + (uint32_t)(kk * 8),
                            vd + (uint64_t)(kk * v_step), idesc_o, (accumulate || kk > 0) ? 1u : 0u);
          mma_commit_warp(bar_pv_done + 8 * t);
          issued = true;
        };
        if (n > 0) {
          if (!ensure_kv(kvc)) break;
          issue_s(kvc);
          clean_v(kvc, 0);
        }
        for (int j = 0; j < n_kv && ok; ++j) {
          const long kv_j = kvc + j;
          if (j < n) {
            // Next scores as soon as the softmax threads have read S(j) (s_free).
            if (!SM::P_ALIAS && j + 1 < n) {
              if (!wait(bar_s_free + 8 * t, (uint32_t)(sfc++ & 1))) break;
              if (!ensure_kv(kv_j + 1)) break;
              issue_s(kv_j + 1);
              clean_v(kv_j + 1, j + 1);
            }
            if (!wait(bar_p_full + 8 * t, (uint32_t)(pc++ & 1))) break;
            // The first P V of an item overwrites O: the previous item's O must be read.
            if (j == 0 && !wait(bar_o_free + 8 * t, (uint32_t)(oc++ & 1) ^ 1u)) break;
            issue_pv(kv_j, j > 0);
            if (j + 1 == n) mma_commit_warp(bar_o_full + 8 * t);
            mma_commit_warp(bar_kv_empty + 8 * (int)(kv_j % STAGES));
            if (SM::P_ALIAS) {
              // The next S of this tile (S(j+1), or S(0) of the next item) overwrites
              // P(j): P V(j) must have completed.  Every P V is waited for here, in
              // order, so completion pvc of pv_done is unambiguous.
              if (!wait(bar_pv_done + 8 * t, (uint32_t)(pvc & 1))) break;
              if (j + 1 < n) {
                if (!ensure_kv(kv_j + 1)) break;
                issue_s(kv_j + 1);
                clean_v(kv_j + 1, j + 1);
              }
            }
            ++pvc;
          } else {
            // Not used by this query tile: release it once it has landed.
            if (!ensure_kv(kv_j)) break;
            if (lane == 0) mbar_arrive(bar_kv_empty + 8 * (int)(kv_j % STAGES));
            __syncwarp();
          }
        }
        if (!ok) break;
        kvc += n_kv;
        mma_commit_warp(bar_q_empty + 8 * qb);
      }
      if (!ok) {
        if (lane == 0) {
          *abort_flag = 1;
          report_status(p.status, TTTJ_DEV_TIMEOUT_ATTN);
        }
        if (issued) {
          mma_commit_warp(bar_drain + 8 * t);
          mbar_wait(bar_drain + 8 * t, 0, nullptr, limit);
        }
      }
    }
  } else if (warp < 4 * NT) {
    // ------------------------------------------------------------ softmax, warps 0-7
    const int t = warp >> 2;             // query tile of this warpgroup
    const int quad = warp & 3;           // TMEM lane quadrant = rows 32*quad..
    const int row = quad * 32 + lane;    // row inside the query tile
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + (t == 0 ? SM::TMEM_S0 : SM::TMEM_S1);
    const uint32_t p_addr = tmem + lane_base + (t == 0 ? SM::TMEM_P0 : SM::TMEM_P1);
    const uint32_t o_addr = tmem + lane_base + (t == 0 ? SM::TMEM_O0 : SM::TMEM_O1);
    const float scale = p.scale_log2;
    long sc = 0, ofc = 0;
    long pv_before = 0;  // P V MMAs of this tile issued before the current item
    bool ok = true;
    int k = 0;
    for (; ok; ++k) {
      const int qb = k % QBUF;
      if (!mbar_wait(bar_q_full + 8 * qb, (uint32_t)((k / QBUF) & 1), abort_flag, limit)) {
        ok = false;
        break;
      }
      // The item's fields as scalars (a copy of the whole struct, indexed by the
      // run-time tile, would live in local memory).
      const AtcItem& wi = info[qb];
      if (wi.n_kv < 0) break;  // no more items
      const int tq = atc_query_tile<NT>(t, k);  // query tile of this item on this side
      const int n = tq == 0 ? wi.n[0] : wi.n[1];
      const int kv_end = tq == 0 ? wi.kv_end[0] : wi.kv_end[1];
      struct {
        int seq0, len, q0, h;
      } w = {wi.seq0, wi.len, wi.q0, wi.h};
      mbar_arrive(bar_q_empty + 8 * qb);  // this thread no longer needs the info slot
      if (n == 0) continue;
      const int qrow = w.q0 + tq * ATC_BM + row;  // query index inside the sequence
      float m_run = -INFINITY;  // running max (log2 domain) used as the exp base
      float l_run = 0.f;
      for (int j = 0; j < n; ++j) {
        if (!mbar_wait(bar_s_full + 8 * t, (uint32_t)(sc++ & 1), abort_flag, limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sv[ATC_BN];  // raw fp32 scores of this thread's row
#pragma unroll
        for (int c = 0; c < ATC_BN / 32; ++c) {
          uint32_t chunk[32];
          tmem_ld_32x32b_x32(s_addr + (uint32_t)(c * 32), chunk);
#pragma unroll
          for (int e = 0; e < 32; ++e) sv[c * 32 + e] = chunk[e];
        }
        tmem_wait_ld();
        // The scores are in registers: the S buffer may take the next tile's scores.
        if (!SM::P_ALIAS && j + 1 < n) {
          tc_fence_before();
          mbar_arrive(bar_s_free + 8 * t);
        }
        const int k0 = j * ATC_BN;
        const bool need_mask =
            (k0 + ATC_BN > kv_end) || (CAUSAL && k0 + ATC_BN - 1 > w.q0 + tq * ATC_BM);
        if (need_mask) {
          // Column c of this tile is masked when c > lim (key >= kv_end, or key > query).
          const int lim = (CAUSAL ? min(kv_end - 1, qrow) : kv_end - 1) - k0;
#pragma unroll
          for (int c = 0; c < ATC_BN; ++c)
            if (c > lim) sv[c] = __float_as_uint(-INFINITY);
        }
        // Row max: 8 independent chains of three-input maxima.
        float pm[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pm[i] = __uint_as_float(sv[i]);
#pragma unroll
        for (int c = 8; c < ATC_BN; c += 2)
          pm[(c >> 1) & 7] =
              fmax3f(pm[(c >> 1) & 7], __uint_as_float(sv[c]), __uint_as_float(sv[c + 1]));
        const float mx = fmax3f(fmax3f(pm[0], pm[1], pm[2]), fmax3f(pm[3], pm[4], pm[5]),
                                fmaxf(pm[6], pm[7]));
        const float m_tile = mx * scale;
        float alpha = 1.f;
        bool rescale = false;
        if (j == 0) {
          m_run = m_tile;
        } else {
          // Lazy rescale: keep the old base unless the max grew by more than 2^8.  Only
          // this sequence's query rows vote (rows past its end belong to the next one).
          const bool grow = qrow < w.len && m_tile > m_run + 8.0f;
          if (__any_sync(0xffffffff, grow)) {
            const float m_new = fmaxf(m_run, m_tile);
            alpha = (m_run == -INFINITY) ? 0.f : ex2_approx(m_run - m_new);
            m_run = m_new;
            rescale = true;  // warp-uniform
          }
        }
        const float base = (m_run == -INFINITY) ? 0.f : m_run;
        const float2 sc2 = make_float2(scale, scale), nb2 = make_float2(-base, -base);
        unsigned long long ps2[2] = {0ull, 0ull};  // partial row sums, f32x2 pairs
        // P as fp16 pairs (128 keys -> 64 packed registers, each replacing two scores),
        // in four chunks of 16 pairs; the first ATC_P_EARLY chunks are computed before
        // waiting for the previous P V, so their exponentials overlap it, the rest after
        // it, each stored as soon as it is ready (fewer live registers).  One pair in
        // four takes its exponentials from the FMA pipe (exp2_fma2): the MUFU (16 per
        // clock per SM) is the tighter resource at head_dim 64.
        uint32_t pk[4][16];
        auto exp_chunk = [&](int q) {
#pragma unroll
          for (int cc = 0; cc < 16; ++cc) {
            const int c = q * 16 + cc;
            const float2 x = ffma2(make_float2(__uint_as_float(sv[2 * c]), __uint_as_float(sv[2 * c + 1])),
                                   sc2, nb2);
            float p0, p1;
            if ((c & 3) == 3) {
              const float2 e = exp2_fma2(x);
              p0 = e.x;
              p1 = e.y;
            } else {
              p0 = ex2_approx(x.x);
              p1 = ex2_approx(x.y);
            }
            ps2[c & 1] = add2p(ps2[c & 1], pk2(p0, p1));
            pk[q][cc] = pack_half2(p0, p1);
          }
        };
#pragma unroll
        for (int q = 0; q < ATC_P_EARLY; ++q) exp_chunk(q);
        // P(j) replaces P(j-1) in the P buffer, and O is rescaled below: P V(j-1) must
        // be complete.  (It was issued when this thread published P(j-1); completion
        // number pv_before + j - 1 of pv_done.  P V(j) cannot exist yet, and completion
        // j - 2 (or the previous item's last, via o_full) was observed already, so the
        // parity is unambiguous.)  At j == 0 the previous item's o_full covered it.
        // With P written over S (head_dim >= 128), s_full(j) already implies it.
        if (!SM::P_ALIAS && j > 0) {
          if (!mbar_wait(bar_pv_done + 8 * t, (uint32_t)((pv_before + j - 1) & 1), abort_flag,
                         limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (q >= ATC_P_EARLY) exp_chunk(q);
          tmem_st_32x32b_x16(p_addr + (uint32_t)(q * 16), pk[q]);
        }
        const float2 rs2 = upk2(add2p(ps2[0], ps2[1]));
        l_run = l_run * alpha + (rs2.x + rs2.y);
        if (rescale) {
          // O holds P V of the key tiles < j (complete, see above): scale it in place.
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(o_addr + (uint32_t)(c * 32), o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st_32x32b_x32(o_addr + (uint32_t)(c * 32), o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar_p_full + 8 * t);
      }
      pv_before += n;
      if (!ok) break;
      // Epilogue: O / l for the valid rows.
      if (!mbar_wait(bar_o_full + 8 * t, (uint32_t)(ofc++ & 1), abort_flag, limit)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      if constexpr (SM::STAGED_EPI) {
        // The warp's 32 rows go through shared memory so that the stores to ctx cover
        // whole row segments (16-byte chunk j of row r staged at slot j ^ (r % NCH));
        // rows past the sequence end are never written (they belong to the next
        // sequence of the packed layout).
        constexpr int NCH = SM::EPI_ROW / 16;  // 16-byte chunks per row
        const uint32_t stage = sEpi + (uint32_t)(warp * 32 * SM::EPI_ROW);
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(o_addr + (uint32_t)(c * 32), o);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int j = c * 4 + q;  // 8 halves = one 16-byte chunk
            const uint32_t a = stage + (uint32_t)(lane * SM::EPI_ROW + ((j ^ (lane % NCH)) << 4));
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a),
                         "r"(pack_half2(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv)),
                         "r"(pack_half2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv)),
                         "r"(pack_half2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv)),
                         "r"(pack_half2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv))
                         : "memory");
          }
        }
        __syncwarp();
        {
          constexpr int RPI = 32 / NCH;  // rows per store instruction
          const int j = lane % NCH;
          const int q0row = w.q0 + tq * ATC_BM + quad * 32;  // first query row of this warp
#pragma unroll
          for (int it = 0; it < 32 / RPI; ++it) {
            const int rr = it * RPI + lane / NCH;
            const uint32_t a = stage + (uint32_t)(rr * SM::EPI_ROW + ((j ^ (rr % NCH)) << 4));
            uint4 v;
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                         : "r"(a)
                         : "memory");
            const int qr = q0row + rr;
            if (qr < w.len && w.seq0 + qr < p.rows_max)
              *reinterpret_cast<uint4*>(p.ctx + (size_t)(w.seq0 + qr) * W + w.h * HD + j * 8) = v;
          }
        }
      } else {
        // Wide heads: each thread stores its own row, 64 bytes per 32 columns.
        const int qr = w.q0 + tq * ATC_BM + row;
        const bool store = qr < w.len && w.seq0 + qr < p.rows_max;
        __half* dst = p.ctx + (size_t)(w.seq0 + qr) * W + w.h * HD;
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(o_addr + (uint32_t)(c * 32), o);
          tmem_wait_ld();
          if (store) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4*>(dst + c * 32 + q * 8) = make_uint4(
                  pack_half2(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv),
                  pack_half2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv),
                  pack_half2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv),
                  pack_half2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv));
          }
        }
      }
      __syncwarp();
      tc_fence_before();
      mbar_arrive(bar_o_free + 8 * t);
    }
    if (!ok) {
      *abort_flag = 1;
      report_status(p.status, TTTJ_DEV_TIMEOUT_ATTN);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace tttj
