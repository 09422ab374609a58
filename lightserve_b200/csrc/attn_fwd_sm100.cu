// FlashAttention forward on the 5th-generation tensor cores (sm_100a).
//
// Same arithmetic as lightserve's _flash_attn_fwd_kernel /
// _flash_attn_fwd_lse_kernel (kernels/flash_attention.py:84-179,
// kernels/flash_attention_backward.py:88-169): S = Q K^T * scale with the
// causal and sequence-end masks, online softmax with fp32 row statistics,
// P rounded to the input dtype before P V, O = acc / l, L = m + ln(l).
//
// B200 design: a persistent kernel, one CTA per SM. A work item is 256 query
// rows (two tiles of 128) of one (batch, head); CTAs take items from a
// global counter in slice-group order (groups of BH_GROUP (batch, head)
// slices; inside a group the longest causal items first), so the slices in
// flight share K / V in L2 and every SM stays busy to the end.
//  * warp 2: work fetcher: takes item ids from the counter and decodes them
//    up to NIS items ahead into a shared-memory ring.
//  * warp 0: TMA producer. Q tiles per item (each tile as
//    soon as the previous item's last QK on it is done), K and V tiles of
//    128 keys through a 2-stage ring that runs on across items.
//  * warp 1: TMEM owner and single-thread MMA issuer. Two query tiles share
//    each K/V tile: S_t = Q_t K^T (SS MMA, fp32 in TMEM) and O_t += P_t V
//    (TS MMA: P read from TMEM, V from shared memory).
//  * warpgroups 1 and 2: softmax for query tile 0 and 1, one thread per row
//    (TMEM lane). Each thread loads its 128 scores with tcgen05.ld, takes the
//    row max, exponentiates with ex2 on log2(e)-prescaled scores, writes P as
//    packed 16-bit pairs over the first 64 columns of its S buffer in two
//    halves (keys [0,64) then [64,128), each with its own p_full barrier, so
//    the first half's PV MMAs overlap the second half's exponentials), and
//    rescales O in TMEM only when the running max grew by more than 2^8
//    (otherwise the stale max is kept; values stay within fp32/bf16 range).
//    At the end of an item the warpgroup normalises and stores its O rows
//    and LSE, then starts the next item; that item's first PV overwrites O
//    only after this warpgroup's p_full, so the read-out needs no barrier.
//  * TMEM: S0 [0,128), S1 [128,256), O0 [256,384), O1 [384,512) columns.
//  * MMA order per K/V tile j: PV_0(j), QK_0(j+1), PV_1(j), QK_1(j+1), so each
//    softmax warpgroup's work overlaps the other tile's two GEMMs;
//    tcgen05.mma instructions of one thread execute in issue order, so
//    QK_t(j+1) may overwrite S_t right after PV_t(j) without a wait.
//  * Every per-(tile, K/V step) barrier completes once per step, so its phase
//    is that tile's running step count across items.
//  * Every mbarrier wait is bounded (sm100.cuh); on a timeout the kernel
//    records an error code, skips the rest of its work, frees TMEM and exits.
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace lsb {

namespace fa_fwd {

constexpr int BM = 128;      // query rows per tile (= TMEM lanes)
constexpr int BN = 128;      // keys per K/V tile
constexpr int TILES = 2;     // query tiles per work item
constexpr int NS = 2;        // K/V ring stages
constexpr int NIS = 4;       // work-item id ring slots
constexpr int THREADS = 384;
constexpr int CHUNK_BYTES = 128 * 128;  // one [128 rows][64 cols] 16-bit box
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units
// (batch, head) slices scheduled together (8 and 32 measured slower or equal).
constexpr int BH_GROUP = 16;
// Variable-length mode with at most this many slice groups and sequences
// enumerates only the items inside sequences (per-sequence block counts and
// a per-group prefix table in shared memory); beyond it, items past a
// sequence's end are fetched and skipped.
constexpr int MAX_TABLE_GROUPS = 128;
constexpr int MAX_TABLE_SEQS = 512;  // per-sequence block counts (uint16) in shared memory

template <int D>
struct Smem {
  static constexpr int KC = D / 64;  // 64-column chunks per row
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + TILES * KC * CHUNK_BYTES;
  static constexpr int V_OFF = K_OFF + NS * KC * CHUNK_BYTES;
  static constexpr int BAR_OFF = V_OFF + NS * KC * CHUNK_BYTES;
  // barriers: q_full[2], q_empty[2], k_full[NS], v_full[NS], kv_empty[NS], s_full[2],
  // p_full[2][2], pv_done[2], item_full[NIS], item_empty[NIS]
  static constexpr int NBAR = 2 * TILES + 3 * NS + 4 * TILES + 2 * NIS + 1;
  static constexpr int TMEM_SLOT_OFF = BAR_OFF + NBAR * 8;
  static constexpr int ITEM_OFF = TMEM_SLOT_OFF + 16;
  static constexpr int TABLE_OFF = ITEM_OFF + NIS * 12;  // ids, then (slice, block) pairs
  static constexpr int SEQ_NB_OFF = TABLE_OFF + (MAX_TABLE_GROUPS + 1) * 4;
  static constexpr int BYTES = SEQ_NB_OFF + MAX_TABLE_SEQS * 2;
  static constexpr int ALLOC = BYTES + 1024;  // slack for 1024-byte alignment
};

struct Params {
  void* o;
  float* lse;
  int* work_counter;  // zeroed before launch; CTAs take work items from it
  // Variable-length mode (non-NULL): sequences packed along the row axis,
  // sequence s = rows [cu_seqlens[s], cu_seqlens[s+1]); "b" is then the
  // sequence index, N the total row count, and LSE is [H, N].
  const int* cu_seqlens;
  int64_t so_b, so_h, so_n;
  int H, N, BH;
  int num_q_ctas;
  float scale_log2;
  int causal;
  int n_groups;  // ceil(BH / BH_GROUP)
  int compact;   // variable-length mode: items from the shared-memory group table
};

// Work-item counters, one per in-flight launch (slot chosen per launch and
// zeroed on the launch stream just before it).
constexpr int COUNTER_SLOTS = 256;
__device__ int g_work_counters[COUNTER_SLOTS];

using namespace sm100;

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 32-byte global store (sm_100 256-bit vector store); dst 32-byte aligned.
__device__ __forceinline__ void st_global_v8(void* dst, const uint32_t* w) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(dst), "r"(w[0]), "r"(w[1]),
               "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

// Row max over a thread's 128 scores (three-input max, 8 independent partial
// maxima for short dependency chains); with MASK, columns >= lim are set to
// -inf first (in place).
template <bool MASK>
__device__ __forceinline__ float row_max(uint32_t (&sr)[4][32], int lim) {
  if (MASK) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int cc = 0; cc < 32; ++cc)
        if (32 * i + cc >= lim) sr[i][cc] = __float_as_uint(-INFINITY);
  }
  float mx8[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) mx8[u] = -INFINITY;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int cc = 0; cc < 32; cc += 2)
      mx8[(cc >> 1) & 7] = max3f(mx8[(cc >> 1) & 7], __uint_as_float(sr[i][cc]),
                                 __uint_as_float(sr[i][cc + 1]));
  return fmaxf(max3f(mx8[0], mx8[1], mx8[2]),
               max3f(max3f(mx8[3], mx8[4], mx8[5]), mx8[6], mx8[7]));
}

// One work item: query rows [q0, q0 + 256) of one (batch, head) slice.
// Rows are slice-relative; `base` is the slice's first row in the tensor
// (its cu_seqlens entry in variable-length mode), `n` its length, `tb` the
// batch coordinate of the TMA maps (0 in variable-length mode).
struct Item {
  int bh, b, h, q0;
  int base, n, tb;
  int nkv_t[TILES];  // K/V tiles each query tile visits (0: tile past the end)
  int nkv;
};
// Rows [base, base + n) of sequence b in variable-length mode, clamped to
// the tensor so malformed offsets cannot reach outside it.
__device__ __forceinline__ void seq_rows(const Params& p, int b, int& base, int& n) {
  base = min(max(__ldg(p.cu_seqlens + b), 0), p.N);
  n = min(max(__ldg(p.cu_seqlens + b + 1), base), p.N) - base;
}

__device__ __forceinline__ void finish_item(Item& w, const Params& p) {
  const int nkv_all = (w.n + BN - 1) / BN;
#pragma unroll
  for (int t = 0; t < TILES; ++t) {
    const int qt0 = w.q0 + t * BM;
    w.nkv_t[t] = qt0 >= w.n ? 0 : (p.causal ? min(nkv_all, qt0 / BN + 1) : nkv_all);
  }
  w.nkv = max(w.nkv_t[0], w.nkv_t[1]);
}

// The item of query block c (rows [256 c, 256 c + 256)) of slice bh.
__device__ __forceinline__ Item make_item(const Params& p, int bh, int c) {
  Item w;
  w.bh = bh;
  w.b = bh / p.H;
  w.h = bh % p.H;
  w.q0 = c * (TILES * BM);
  if (p.cu_seqlens != nullptr) {
    seq_rows(p, w.b, w.base, w.n);
    w.tb = 0;
  } else {
    w.base = 0;
    w.n = p.N;
    w.tb = w.b;
  }
  finish_item(w, p);
  return w;
}

// Items are numbered group by group (BH_GROUP consecutive slices). Dense
// mode: inside a group, block index major (causal: the longest blocks
// first), slice minor. Compact variable-length mode (gtab = items before
// each group): only blocks inside their sequence are numbered; inside a
// group block index c descends and, at each c, the group's slices that
// have a block c follow in slice order.
__device__ __forceinline__ Item decode_item(int item, const Params& p, bool compact,
                                            const int* gtab, const uint16_t* seq_nb) {
  if (compact) {
    // Group: the last g with gtab[g] <= item (binary search).
    int lo = 0, hi = p.n_groups - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (gtab[mid] <= item) lo = mid; else hi = mid - 1;
    }
    const int g = lo;
    const int r = item - gtab[g];
    const int s0 = g * BH_GROUP;
    const int gsz = min(BH_GROUP, p.BH - s0);
    int nb[BH_GROUP];
    int cmax = 0;
    int sq = s0 / p.H, hh = s0 - sq * p.H;  // sequence and head of slice s0 + i
#pragma unroll
    for (int i = 0; i < BH_GROUP; ++i) {
      nb[i] = i < gsz ? (int)seq_nb[sq] : 0;
      cmax = max(cmax, nb[i] - 1);
      if (++hh == p.H) { hh = 0; ++sq; }
    }
    // above(c) = items of the group at block indices > c (non-increasing in
    // c); the item's block index is the smallest c with above(c) <= r.
    auto above = [&](int c) {
      int a = 0;
#pragma unroll
      for (int i = 0; i < BH_GROUP; ++i) a += max(0, nb[i] - 1 - c);
      return a;
    };
    int clo = 0, chi = cmax;
    while (clo < chi) {
      const int mid = (clo + chi) >> 1;
      if (above(mid) <= r) chi = mid; else clo = mid + 1;
    }
    const int c = clo;
    int idx = r - above(c);  // position among the group's slices that have block c
    int sel = 0;
    for (int i = 0; i < gsz; ++i) {
      if (nb[i] > c) {
        if (idx == 0) { sel = i; break; }
        --idx;
      }
    }
    return make_item(p, s0 + sel, c);
  }
  const int nq = p.num_q_ctas;
  const int g = item / (BH_GROUP * nq);
  const int rem = item - g * BH_GROUP * nq;
  const int gsz = min(BH_GROUP, p.BH - g * BH_GROUP);
  const int ci = rem / gsz;
  const int c = p.causal ? (nq - 1 - ci) : ci;  // causal: longest items first
  return make_item(p, g * BH_GROUP + rem % gsz, c);
}

template <int D, int FMT>
__global__ void __launch_bounds__(THREADS, 1)
fa_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
              const __grid_constant__ CUtensorMap tv, const Params p) {
  using L = Smem<D>;
  constexpr int KC = L::KC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* q_full = bars;                     // [TILES]
  uint64_t* q_empty = q_full + TILES;          // [TILES]: the item's last QK on Q_t is done
  uint64_t* k_full = q_empty + TILES;          // [NS]
  uint64_t* v_full = k_full + NS;              // [NS]
  uint64_t* kv_empty = v_full + NS;            // [NS]
  uint64_t* s_full = kv_empty + NS;            // [TILES]
  // [TILES][2]: the P of keys [0, 64) / [64, 128) of the step is in TMEM
  // (the first half's PV MMAs run while the softmax computes the second).
  uint64_t* p_full = s_full + TILES;
  uint64_t* pv_done = p_full + 2 * TILES;      // [TILES]
  uint64_t* item_full = pv_done + TILES;       // [NIS]
  uint64_t* item_empty = item_full + NIS;      // [NIS]: 10 arrivals (TMA, MMA, 8 softmax warps)
  // The TMA producer has reached the last K/V tiles of its current item: the
  // fetcher may claim the next one.
  uint64_t* fetch_go = item_empty + NIS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::TMEM_SLOT_OFF);
  volatile int* item_ids = reinterpret_cast<volatile int*>(smem + L::ITEM_OFF);
  // (slice, block) of each ring slot's item, decoded once by the producer.
  volatile int* item_code = item_ids + NIS;
  int* gtab = reinterpret_cast<int*>(smem + L::TABLE_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint16_t* seq_nb = reinterpret_cast<uint16_t*>(smem + L::SEQ_NB_OFF);
  if (p.compact) {
    // seq_nb[s] = 256-row blocks of sequence s (one load pair per thread);
    // gtab[g] = items of the groups before g: per-group sums, then a prefix
    // sum by warp 0 (shuffle scan over 32 groups at a time).
    const int n_seqs = p.BH / p.H;
    for (int sq = threadIdx.x; sq < n_seqs; sq += THREADS) {
      int base, n;
      seq_rows(p, sq, base, n);
      // At most num_q_ctas blocks (max_seqlen rows), as in the uncompacted
      // numbering.
      seq_nb[sq] = (uint16_t)min((n + TILES * BM - 1) / (TILES * BM), p.num_q_ctas);
    }
    __syncthreads();
    for (int g = threadIdx.x; g < p.n_groups; g += THREADS) {
      const int s0 = g * BH_GROUP, s1 = min(p.BH, s0 + BH_GROUP);
      int cnt = 0;
      for (int bh = s0; bh < s1; ++bh) cnt += seq_nb[bh / p.H];
      gtab[g + 1] = cnt;
    }
    __syncthreads();
    if (warp == 0) {
      int carry = 0;
      if (lane == 0) gtab[0] = 0;
      for (int g0 = 0; g0 < p.n_groups; g0 += 32) {
        const int g = g0 + lane;
        int v = g < p.n_groups ? gtab[g + 1] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int u = __shfl_up_sync(0xffffffffu, v, o);
          if (lane >= o) v += u;
        }
        if (g < p.n_groups) gtab[g + 1] = carry + v;
        carry += __shfl_sync(0xffffffffu, v, 31);
      }
    }
    // The __syncthreads below (after TMEM allocation) publishes the table.
  }
  // Consumer side of the work-item ring: id of the k-th item (>= n_items:
  // no more work), or -1 when the wait gave up; its slice and block index.
  auto next_item = [&](int k, int& bh, int& c) -> int {
    const int slot = k % NIS;
    if (!mbar_wait(&item_full[slot], (k / NIS) & 1, 0x10A)) return -1;
    const int id = item_ids[slot];
    bh = item_code[2 * slot];
    c = item_code[2 * slot + 1];
    mbar_arrive(&item_empty[slot]);
    return id;
  };

  if (threadIdx.x == 0) {
    for (int t = 0; t < TILES; ++t) {
      mbar_init(&q_full[t], 1);
      mbar_init(&q_empty[t], 1);
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[2 * t], BM);
      mbar_init(&p_full[2 * t + 1], BM);
      mbar_init(&pv_done[t], 1);
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < NIS; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 10);
    }
    mbar_init(fetch_go, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // The compact numbering pays for its longer decoding only when it drops
  // more than an eighth of the items (every CTA decides alike).
  const int n_all = p.BH * p.num_q_ctas;
  const bool compact = p.compact && (int64_t)gtab[p.n_groups] * 8 < (int64_t)n_all * 7;
  const int n_items = compact ? gtab[p.n_groups] : n_all;

  uint8_t* sQ = smem + L::Q_OFF;
  uint8_t* sK = smem + L::K_OFF;
  uint8_t* sV = smem + L::V_OFF;

  // Register split: 384 threads x 168 at launch >= 128 x 96 (TMA/MMA
  // warpgroup) + 256 x 200 (softmax warpgroups).
  // (setmaxnreg sits at the top of each role's branch so ptxas budgets each.)
  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    reg_dealloc<96>();
    if (lane == 0) {
      prefetch_tmap(&tq); prefetch_tmap(&tk); prefetch_tmap(&tv);
      int J = 0;  // running K/V tile count of this CTA
      bool ok = true;
      for (int k = 0; ok; ++k) {
        int ibh = 0, ic = 0;
        const int item = next_item(k, ibh, ic);
        if (item < 0 || item >= n_items) break;
        const Item w = make_item(p, ibh, ic);
        for (int t = 0; t < TILES; ++t) {
          if (k > 0 && !mbar_wait(&q_empty[t], (k - 1) & 1, 0x103)) { ok = false; break; }
          if (w.nkv_t[t] == 0) {  // tile past the slice end: nothing to load
            mbar_arrive(&q_full[t]);
            continue;
          }
          mbar_arrive_expect_tx(&q_full[t], KC * CHUNK_BYTES);
          for (int kc = 0; kc < KC; ++kc)
            tma_load_4d(sQ + (t * KC + kc) * CHUNK_BYTES, &tq, &q_full[t], kc * 64,
                        w.base + w.q0 + t * BM, w.h, w.tb);
        }
        // Claim point of the next item: four K/V tiles before the end of this
        // one (its start for items of at most four tiles), close to the end
        // of this item's compute, so the items left at the end of the
        // launch stay unclaimed until an SM is about to need one, while the
        // claim and its decoding still finish before the producer needs it.
        const int go_at = max(w.nkv - 4, 0);
        if (go_at == 0) mbar_arrive(fetch_go);
        for (int j = 0; ok && j < w.nkv; ++j, ++J) {
          if (j == go_at && j > 0) mbar_arrive(fetch_go);
          const int s = J % NS;
          if (J >= NS && !mbar_wait(&kv_empty[s], ((J / NS) - 1) & 1, 0x101)) { ok = false; break; }
          mbar_arrive_expect_tx(&k_full[s], KC * CHUNK_BYTES);
          for (int kc = 0; kc < KC; ++kc)
            tma_load_4d(sK + (s * KC + kc) * CHUNK_BYTES, &tk, &k_full[s], kc * 64,
                        w.base + j * BN, w.h, w.tb);
          mbar_arrive_expect_tx(&v_full[s], KC * CHUNK_BYTES);
          for (int kc = 0; kc < KC; ++kc)
            tma_load_4d(sV + (s * KC + kc) * CHUNK_BYTES, &tv, &v_full[s], kc * 64,
                        w.base + j * BN, w.h, w.tb);
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issue --
    reg_dealloc<96>();
    if (lane == 0) {
      constexpr uint32_t IDESC_QK = idesc_f16(BM, BN, FMT, 0, 0);
      constexpr uint32_t IDESC_PV = idesc_f16(BM, D, FMT, 0, 1);
      const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK), v_base = smem_u32(sV);
      auto issue_qk = [&](int t, int J) {
        const int s = J % NS;
        const uint32_t d_tmem = tmem + t * 128;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk / 4) * CHUNK_BYTES + (kk % 4) * 32;
          const uint64_t a = smem_desc_sw128(q_base + (t * KC) * CHUNK_BYTES + off, 16, 1024);
          const uint64_t bd = smem_desc_sw128(k_base + (s * KC) * CHUNK_BYTES + off, 16, 1024);
          mma_ss(d_tmem, a, bd, IDESC_QK, kk > 0);
        }
        mma_commit(&s_full[t]);
      };
      // PV over keys [64 h, 64 h + 64) of the K/V tile (K-steps 4h .. 4h+3);
      // the second half commits pv_done.
      auto issue_pv_half = [&](int t, int J, bool acc, int h) {
        const int s = J % NS;
        const uint32_t d_tmem = tmem + 256 + t * 128;
#pragma unroll
        for (int k4 = 0; k4 < BN / 32; ++k4) {
          const int kk = h * (BN / 32) + k4;
          const uint64_t bd =
              smem_desc_sw128(v_base + (s * KC) * CHUNK_BYTES + kk * 2048, CHUNK_BYTES, 1024);
          mma_ts(d_tmem, tmem + t * 128 + kk * 8, bd, IDESC_PV, (acc || kk > 0) ? 1u : 0u);
        }
        if (h == 1) mma_commit(&pv_done[t]);
      };
      int J = 0;                     // running K/V tile count
      int jt[TILES] = {0, 0};        // running K/V step count per query tile
      bool ok = true;
      for (int k = 0; ok; ++k) {
        int ibh = 0, ic = 0;
        const int item = next_item(k, ibh, ic);
        if (item < 0 || item >= n_items) break;
        const Item w = make_item(p, ibh, ic);
        for (int t = 0; t < TILES && ok; ++t)
          if (!mbar_wait(&q_full[t], k & 1, 0x201)) ok = false;
        if (!ok) break;
        if (w.nkv > 0 && !mbar_wait(&k_full[J % NS], (J / NS) & 1, 0x202)) { ok = false; break; }
        tc_fence_after();
        for (int t = 0; t < TILES; ++t) {
          if (w.nkv_t[t] > 0) issue_qk(t, J);
          if (w.nkv_t[t] <= 1) mma_commit(&q_empty[t]);  // last (or no) QK on Q_t
        }
        for (int j = 0; ok && j < w.nkv; ++j) {
          const int s = (J + j) % NS;
          if (!mbar_wait(&v_full[s], ((J + j) / NS) & 1, 0x203)) { ok = false; break; }
          for (int t = 0; t < TILES; ++t) {
            if (j >= w.nkv_t[t]) continue;
            // PV_t(0) of an item overwrites O_t: its softmax warpgroup read
            // the previous item's O_t out before this p_full.
            if (!mbar_wait(&p_full[2 * t], (jt[t] + j) & 1, 0x204)) { ok = false; break; }
            tc_fence_after();
            issue_pv_half(t, J + j, j > 0, 0);
            if (!mbar_wait(&p_full[2 * t + 1], (jt[t] + j) & 1, 0x206)) { ok = false; break; }
            tc_fence_after();
            issue_pv_half(t, J + j, j > 0, 1);
            if (j + 1 < w.nkv_t[t]) {
              const int s1 = (J + j + 1) % NS;
              if (!mbar_wait(&k_full[s1], ((J + j + 1) / NS) & 1, 0x205)) { ok = false; break; }
              tc_fence_after();
              issue_qk(t, J + j + 1);
              if (j + 2 == w.nkv_t[t]) mma_commit(&q_empty[t]);  // last QK on Q_t
            }
          }
          mma_commit(&kv_empty[s]);
        }
        J += w.nkv;
        for (int t = 0; t < TILES; ++t) jt[t] += w.nkv_t[t];
      }
    }
  } else if (warp == 2) {
    // -------------------------------------------------------- work fetcher --
    // Takes item ids from the global counter and decodes them into the ring,
    // one item ahead of the TMA producer (claimed when the producer signals
    // fetch_go), so neither the counter's latency nor the decoding sits on
    // the producer's path.
    reg_dealloc<96>();
    if (lane == 0) {
      for (int k = 0;; ++k) {
        const int slot = k % NIS;
        if (k >= NIS && !mbar_wait(&item_empty[slot], ((k / NIS) - 1) & 1, 0x104)) break;
        if (k > 0 && !mbar_wait(fetch_go, (k - 1) & 1, 0x105)) break;
        const int item = atomicAdd(p.work_counter, 1);
        if (item < n_items) {
          const Item w = decode_item(item, p, compact, gtab, seq_nb);
          item_code[2 * slot] = w.bh;
          item_code[2 * slot + 1] = w.q0 / (TILES * BM);
        }
        item_ids[slot] = item;
        mbar_arrive(&item_full[slot]);  // release: the item is visible to its waiters
        if (item >= n_items) break;
      }
    }
  } else if (warp < 4) {
    reg_dealloc<96>();  // warp 3: idle member of the TMA/MMA warpgroup
  } else {
    // ------------------------------------------------------------- softmax --
    reg_alloc<200>();
    const int t = (warp >> 2) - 1;
    const int row = threadIdx.x - 128 * (t + 1);          // TMEM lane of this thread
    const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const float sl2 = p.scale_log2;
    int jt = 0;  // running K/V step count of this query tile
    bool ok = true;
    for (int k = 0; ok; ++k) {
      int item = 0, ibh = 0, ic = 0;
      if (lane == 0) item = next_item(k, ibh, ic);
      item = __shfl_sync(0xffffffffu, item, 0);
      ibh = __shfl_sync(0xffffffffu, ibh, 0);
      ic = __shfl_sync(0xffffffffu, ic, 0);
      if (item < 0 || item >= n_items) break;
      const Item w = make_item(p, ibh, ic);
      const int nkv_t = w.nkv_t[t];
      const int qt0 = w.q0 + t * BM;
      const int row_g = qt0 + row;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < nkv_t; ++j) {
        if (!mbar_wait_warp(&s_full[t], (jt + j) & 1, 0x301)) { ok = false; break; }
        tc_fence_after();
        uint32_t sr[4][32];
#pragma unroll
        for (int i = 0; i < 4; ++i) tmem_ld32(lane_addr + t * 128 + 32 * i, sr[i]);
        tmem_ld_wait();
        const int kv0 = j * BN;
        // Only the diagonal tile (causal) and the tile holding the slice's last
        // key need masks (in variable-length mode that tile's columns past
        // the end hold the next sequence's keys).
        const bool need_mask = (kv0 + BN > w.n) || (p.causal && kv0 + BN - 1 > qt0);
        const int lim = min(w.n, p.causal ? row_g + 1 : w.n) - kv0;  // valid columns < lim
        const float mx = need_mask ? row_max<true>(sr, lim) : row_max<false>(sr, lim);
        const float m_new = fmaxf(m, mx * sl2);
        float alpha = 1.f;
        const bool rescale = m_new > m + RESCALE_THRESHOLD;
        if (rescale) {
          alpha = ex2(m - m_new);
          m = m_new;
          l *= alpha;
        }
        const float m_use = (m == -INFINITY) ? 0.f : m;
        // Packed f32x2 arithmetic halves the instruction count of the scale and
        // row-sum steps; the exponentials go to MUFU.EX2. P is handed over in
        // two halves (keys [0, 64), then [64, 128)), so the MMA thread runs
        // the first half's PV while the second half is exponentiated.
        float2 l2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                        make_float2(0.f, 0.f)};
        const float2 sl2_2 = make_float2(sl2, sl2), negm2 = make_float2(-m_use, -m_use);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int i = 2 * h; i < 2 * h + 2; ++i) {
            uint32_t pk[16];
#pragma unroll
            for (int cc = 0; cc < 16; ++cc) {
              const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[i][2 * cc]),
                                                      __uint_as_float(sr[i][2 * cc + 1])),
                                          sl2_2, negm2);
              const float2 pp = make_float2(ex2(x.x), ex2(x.y));
              l2[cc & 3] = __fadd2_rn(l2[cc & 3], pp);
              pk[cc] = FMT == 1 ? pack_bf16(pp.x, pp.y) : pack_f16(pp.x, pp.y);
            }
#pragma unroll
            for (int cc = 0; cc < 16; ++cc) sr[h][(i & 1) * 16 + cc] = pk[cc];
          }
          tmem_st32(lane_addr + t * 128 + 32 * h, sr[h]);
          // O is rescaled before the first half's PV accumulates into it.
          // tcgen05.ld/st are warp-collective: if any row of the warp
          // rescales, the whole warp runs the loop (alpha is 1 for rows that
          // do not). PV_t(j-1) has completed: s_full(j) follows it in issue
          // order.
          if (h == 0 && __any_sync(0xffffffffu, rescale && j > 0)) {
            const float a = (rescale && j > 0) ? alpha : 1.f;
#pragma unroll
            for (int i = 0; i < D / 32; ++i) {
              uint32_t ov[32];
              tmem_ld32(lane_addr + 256 + t * 128 + 32 * i, ov);
              tmem_ld_wait();
#pragma unroll
              for (int cc = 0; cc < 32; ++cc) ov[cc] = __float_as_uint(__uint_as_float(ov[cc]) * a);
              tmem_st32(lane_addr + 256 + t * 128 + 32 * i, ov);
            }
          }
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(&p_full[2 * t + h]);
        }
        {
          const float2 a2 = __fadd2_rn(__fadd2_rn(l2[0], l2[1]), __fadd2_rn(l2[2], l2[3]));
          l += a2.x + a2.y;
        }
      }
      if (!ok) break;
      if (nkv_t > 0) {
        if (!mbar_wait_warp(&pv_done[t], (jt + nkv_t - 1) & 1, 0x302)) { ok = false; break; }
        tc_fence_after();
        const float inv_l = 1.0f / l;
        uint8_t* orow = reinterpret_cast<uint8_t*>(p.o) +
                        2 * (w.tb * p.so_b + w.h * p.so_h + (int64_t)(w.base + row_g) * p.so_n);
        // Whole 32-byte sectors per store when aligned: with one row per
        // thread, 16-byte stores reach about half the SM's write bandwidth.
        const bool st32 = (reinterpret_cast<uintptr_t>(orow) & 31) == 0;
#pragma unroll
        for (int i = 0; i < D / 32; ++i) {
          uint32_t ov[32];
          tmem_ld32(lane_addr + 256 + t * 128 + 32 * i, ov);
          tmem_ld_wait();
          uint32_t pk[16];
#pragma unroll
          for (int cc = 0; cc < 16; ++cc) {
            const float a0 = __uint_as_float(ov[2 * cc]) * inv_l;
            const float a1 = __uint_as_float(ov[2 * cc + 1]) * inv_l;
            pk[cc] = FMT == 1 ? pack_bf16(a0, a1) : pack_f16(a0, a1);
          }
          if (row_g < w.n && st32) {
#pragma unroll
            for (int v8 = 0; v8 < 2; ++v8) st_global_v8(orow + 64 * i + 32 * v8, &pk[8 * v8]);
          } else if (row_g < w.n) {
            uint4* dst = reinterpret_cast<uint4*>(orow + 64 * i);
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4)
              dst[v4] = make_uint4(pk[4 * v4], pk[4 * v4 + 1], pk[4 * v4 + 2], pk[4 * v4 + 3]);
          }
        }
        if (p.lse != nullptr && row_g < w.n) {
          const int64_t li = p.cu_seqlens != nullptr ? (int64_t)w.h * p.N + w.base + row_g
                                                     : (int64_t)w.bh * p.N + row_g;
          p.lse[li] = (m + __log2f(l)) * 0.6931471805599453f;
        }
        tc_fence_before();
      }
      jt += nkv_t;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace fa_fwd


bool attn_fwd_tc_eligible(const void* q, const void* k, const void* v, const void* o, int64_t B,
                          int64_t H, int64_t N, int64_t D, const int64_t* sq, const int64_t* sk,
                          const int64_t* sv, const int64_t* so, int dtype) {
  if (dtype != LSB_DTYPE_BF16 && dtype != LSB_DTYPE_F16) return false;
  if (D != 64 && D != 128) return false;
  if (N >= (1LL << 30) || B * H * ((N + 255) / 256) > 0x7fffffff) return false;
  if (!tma_ok(q, B, H, N, sq, 2) || !tma_ok(k, B, H, N, sk, 2) || !tma_ok(v, B, H, N, sv, 2))
    return false;
  // Output rows are written with 16-byte stores.
  if (!aligned16(o) || so[3] != 1 || (so[2] * 2) % 16 || (so[1] * 2) % 16 || (so[0] * 2) % 16)
    return false;
  return true;
}

// Dense mode: cu_seqlens == NULL, B slices of N rows. Variable-length mode:
// B == 1, N = total rows, n_seqs sequences at cu_seqlens (device), the
// longest max_seqlen rows.
template <int D, int FMT>
static int launch_fa_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                         int64_t B, int64_t H, int64_t N, const int64_t* sq, const int64_t* sk,
                         const int64_t* sv, const int64_t* so, float scale, int causal,
                         int dtype, cudaStream_t st, const int* cu_seqlens = nullptr,
                         int64_t n_seqs = 0, int64_t max_seqlen = 0) {
  using namespace fa_fwd;
  CUtensorMap mq, mk, mv;
  int rc = make_bhnd_map(&mq, q, dtype, B, H, N, D, sq, 64, BM);
  if (!rc) rc = make_bhnd_map(&mk, k, dtype, B, H, N, D, sk, 64, BN);
  if (!rc) rc = make_bhnd_map(&mv, v, dtype, B, H, N, D, sv, 64, BN);
  if (rc) return rc;
  Params p;
  p.o = o; p.lse = lse;
  p.so_b = so[0]; p.so_h = so[1]; p.so_n = so[2];
  p.cu_seqlens = cu_seqlens;
  p.H = (int)H; p.N = (int)N;
  p.BH = (int)((cu_seqlens != nullptr ? n_seqs : B) * H);
  const int64_t rows = cu_seqlens != nullptr ? max_seqlen : N;
  p.num_q_ctas = (int)((rows + TILES * BM - 1) / (TILES * BM));
  p.n_groups = (p.BH + BH_GROUP - 1) / BH_GROUP;
  p.compact = cu_seqlens != nullptr && p.n_groups <= MAX_TABLE_GROUPS && n_seqs <= MAX_TABLE_SEQS &&
              rows <= (int64_t)TILES * BM * 0xffff;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  // Work-item counter: a slot of g_work_counters per launch, zeroed in stream
  // order just before the kernel. Eager launches rotate through the first
  // half of the slots, so launches in flight on other streams use other
  // slots. A launch recorded into a CUDA graph keeps its slot for every
  // replay, so recorded launches take slots from the second half instead and
  // never share one with an eager launch (only 128 or more recorded launches
  // replayed concurrently with each other could collide).
  const int dev = current_device("attn_fwd_tc");
  if (dev < 0) return LSB_ERR_CUDA;
  static int* counters[kMaxDevices] = {nullptr};
  static PerDeviceOnce counter_lookup;
  LSB_CUDA_OK(counter_lookup.run(dev, [&] {
    void* addr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&addr, g_work_counters);
    counters[dev] = static_cast<int*>(addr);
    return e;
  }), "attn_fwd_tc counter symbol");
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  LSB_CUDA_OK(cudaStreamIsCapturing(st, &cap), "attn_fwd_tc capture status");
  static std::atomic<unsigned> next_eager{0}, next_captured{0};
  constexpr unsigned HALF = COUNTER_SLOTS / 2;
  const unsigned slot = cap == cudaStreamCaptureStatusNone
                            ? next_eager.fetch_add(1, std::memory_order_relaxed) % HALF
                            : HALF + next_captured.fetch_add(1, std::memory_order_relaxed) % HALF;
  p.work_counter = counters[dev] + slot;
  LSB_CUDA_OK(cudaMemsetAsync(p.work_counter, 0, sizeof(int), st), "attn_fwd_tc counter reset");
  const int smem = Smem<D>::ALLOC;
  auto kern = fa_fwd_kernel<D, FMT>;
  static SmemLimit smem_limit;
  if (int rc_ = smem_limit.ensure(kern, smem, "attn_fwd_tc smem attribute")) return rc_;
  // Persistent: one CTA per SM (shared memory and TMEM allow no more).
  const int64_t n_items = (int64_t)p.BH * p.num_q_ctas;
  dim3 grid((unsigned)std::min<int64_t>(n_items, num_sms()));
  kern<<<grid, THREADS, smem, st>>>(mq, mk, mv, p);
  LSB_CHECK_LAUNCH("attn_fwd_tc");
  return LSB_OK;
}

int attn_fwd_tc(const void* q, const void* k, const void* v, void* o, float* lse, int64_t B,
                int64_t H, int64_t N, int64_t D, const int64_t* sq, const int64_t* sk,
                const int64_t* sv, const int64_t* so, float scale, int causal, int dtype,
                cudaStream_t st) {
  const bool bf = dtype == LSB_DTYPE_BF16;
  if (D == 128)
    return bf ? launch_fa_fwd<128, 1>(q, k, v, o, lse, B, H, N, sq, sk, sv, so, scale, causal, dtype, st)
              : launch_fa_fwd<128, 0>(q, k, v, o, lse, B, H, N, sq, sk, sv, so, scale, causal, dtype, st);
  return bf ? launch_fa_fwd<64, 1>(q, k, v, o, lse, B, H, N, sq, sk, sv, so, scale, causal, dtype, st)
            : launch_fa_fwd<64, 0>(q, k, v, o, lse, B, H, N, sq, sk, sv, so, scale, causal, dtype, st);
}

int attn_fwd_varlen_tc(const void* q, const void* k, const void* v, void* o, float* lse,
                       const int* cu_seqlens, int64_t n_seqs, int64_t max_seqlen, int64_t T,
                       int64_t H, int64_t D, const int64_t* sq, const int64_t* sk,
                       const int64_t* sv, const int64_t* so, float scale, int causal, int dtype,
                       cudaStream_t st) {
  // [T, H, D] with strides {token, head, 1} as a [1, H, T, D] tensor.
  const int64_t q4[4] = {0, sq[1], sq[0], 1}, k4[4] = {0, sk[1], sk[0], 1};
  const int64_t v4[4] = {0, sv[1], sv[0], 1}, o4[4] = {0, so[1], so[0], 1};
  const bool bf = dtype == LSB_DTYPE_BF16;
  if (D == 128)
    return bf ? launch_fa_fwd<128, 1>(q, k, v, o, lse, 1, H, T, q4, k4, v4, o4, scale, causal, dtype,
                                      st, cu_seqlens, n_seqs, max_seqlen)
              : launch_fa_fwd<128, 0>(q, k, v, o, lse, 1, H, T, q4, k4, v4, o4, scale, causal, dtype,
                                      st, cu_seqlens, n_seqs, max_seqlen);
  return bf ? launch_fa_fwd<64, 1>(q, k, v, o, lse, 1, H, T, q4, k4, v4, o4, scale, causal, dtype, st,
                                   cu_seqlens, n_seqs, max_seqlen)
            : launch_fa_fwd<64, 0>(q, k, v, o, lse, 1, H, T, q4, k4, v4, o4, scale, causal, dtype, st,
                                   cu_seqlens, n_seqs, max_seqlen);
}

int attn_fwd_tc_device_error(bool reset) {
  return sm100::tu_device_error(reset);
}

}  // namespace lsb
