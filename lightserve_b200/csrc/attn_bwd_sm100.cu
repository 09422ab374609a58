// FlashAttention backward on the 5th-generation tensor cores (sm_100a).
//
// Same arithmetic as lightserve's recomputation backward
// (kernels/flash_attention_backward.py:202-330): Dsum = rowsum(dO * O) (fp32,
// computed by a separate pass); per K/V tile, a sweep over Q tiles that
// recomputes P = exp(S * scale - L) with the forward's log-sum-exp, then
// dV += P^T dO (P rounded to the input dtype), dP = dO V^T,
// dS = P * (dP - Dsum) (rounded to the input dtype), dK += dS^T Q * scale and
// dQ += dS K * scale accumulated in an fp32 buffer, rounded at the end.
//
// B200 design: one CTA per 128 keys of one (batch, head), looping over query
// tiles of 128 rows (causal: starting at the diagonal). Every GEMM is issued
// as M=128, N=128 tcgen05.mma instructions: a tcgen05.mma costs about the same
// time for N=64 as for N=128, so 64-wide tiles would halve the tensor-core
// throughput. Everything is computed transposed so the 128 keys are the TMEM
// lanes; TMEM (512 columns) holds
//   [0,128)   dV  += P^T dO    (TS MMA: P^T packed to 16 bits inside S^T)
//   [128,256) dK  += dS^T Q    (TS MMA: dS^T packed inside S^T)
//   [256,384) S^T  = K Q^T     (SS MMA), then P^T and dS^T in 16-bit pairs
//   [384,512) dP^T = V dO^T    (SS MMA), then dQ^T = K^T dS^T (SS MMA, K^T
//             read MN-major from the K tile, dS^T from a 128-byte-swizzled
//             shared tile)
// Warp 0 streams K/V once per item (V reloaded once the item's last dP^T is
// done, K once its last dQ^T is done, both prefetched into L2 when the item
// is claimed during the previous item's last tile), Q tiles (plus each tile's log-sum-exp and Dsum)
// through a 2-stage ring and dO tiles through one buffer (dO(i+1) loads
// while dQ(i), dK(i) and S(i+1) run); warp 1 owns TMEM and issues the MMAs
// in the order dV(i), dQ(i), dK(i), S(i+1), dP(i+1); warp 2 adds the finished
// dQ tile into the fp32 dQ buffer with two bulk shared->global reductions.
// Warpgroups 1 and 2 split every tile's 128 query columns (64 each): thread =
// key for P^T / dS^T, thread = head-dim index for dQ^T. Once dQ^T(i) is in
// registers, warpgroup 1 stages its 64 query rows in a dedicated 32 KiB
// buffer and warpgroup 2 in the dS^T tile (free after dQ^T(i)). The fp32
// reduction into L2 runs at about 21 B/clk per SM with every SM reducing,
// so the 64 KiB of one tile takes ~3100 cycles: the reductions of tile i
// overlap all of tile i+1's work, and only the next dS^T write waits for
// the dS^T-tile half to have been read.
// All mbarrier waits are bounded (sm100.cuh).
#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace lsb {

struct Strides4 {
  int64_t b, h, n, d;
};
template <typename T>
int launch_dsum(const void* o, const void* dout, float* dsum, int64_t B, int64_t H, int64_t N,
                int64_t D, Strides4 so, Strides4 sdo, cudaStream_t st, float* zero_rows,
                int* zero_counter, bool* zeroed);
template <typename T>
int launch_dq_cast(const float* dq_acc, void* dq, int64_t B, int64_t H, int64_t N, int64_t D,
                   Strides4 sdq, cudaStream_t st);

namespace fa_bwd {

using namespace sm100;

constexpr int BN = 128;   // keys per CTA (TMEM lanes)
constexpr int BM = 128;   // query rows per inner tile
constexpr int THREADS = 384;
constexpr int CHUNK = 128 * 128;  // [128 rows][64 cols] 16-bit box, 128-byte swizzle
constexpr int NQS = 2;            // Q / statistics ring stages
constexpr int STAGE_ROWS = 64;    // dQ rows per staging buffer
constexpr int NIS = 4;            // work-item id ring slots
// k_full, v_full, k_empty, q_full[NQS], q_empty[NQS], stat_full[NQS], do_full, do_empty,
// s_ready, p_ready, dp_ready, ds_ready, dq_ready, dq_free, dk_done, red_full[2],
// red_free[2], epi_staged, epi_v_free, vdo_issued, epi_q_free[NQS], item_full[NIS],
// item_empty[NIS]
constexpr int NBAR = 3 + 4 * NQS + 16 + 2 * NIS;

// Shared-memory plan for head dim D (64 or 128): K, V, NQS Q tiles and dO
// (D / 64 chunks each), the dS^T tile (two 64-query chunks, also dQ staging
// 1), dQ staging 0 (64 rows x D fp32), the per-stage statistics, barriers.
template <int D_>
struct Layout {
  static constexpr int D = D_;
  static constexpr int KC = D / 64;        // chunks per K, V, Q or dO tile
  static constexpr int TILE = KC * CHUNK;
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = K_OFF + TILE;  // directly after K (see the dQ^T MMA)
  static constexpr int Q_OFF = V_OFF + TILE;
  static constexpr int DO_OFF = Q_OFF + NQS * TILE;
  static constexpr int DS_OFF = DO_OFF + TILE;
  static constexpr int STG_OFF = DS_OFF + 2 * CHUNK;
  static constexpr int STAT_OFF = STG_OFF + STAGE_ROWS * D * 4;
  static constexpr int BAR_OFF = STAT_OFF + NQS * 2 * BM * 4;
  static constexpr int SLOT_OFF = BAR_OFF + NBAR * 8;
  static constexpr int ITEM_OFF = SLOT_OFF + 16;  // [NIS] work-item ids
  static constexpr int SMEM = ITEM_OFF + NIS * 4;
  static_assert(STAGE_ROWS * D * 4 <= 2 * CHUNK, "dQ staging 1 lives in the dS^T tile");
  static_assert(SMEM <= 232448, "backward tile set exceeds the 227 KiB shared-memory limit");
};

constexpr uint32_t T_DV = 0, T_DK = 128, T_S = 256, T_DP = 384;
constexpr int BH_GROUP = 16;  // (batch, head) slices scheduled together

struct Params {
  const float* lse;
  const float* dsum;
  float* dq_acc;
  int* work_counter;  // zeroed before launch; CTAs take work items from it
  int H, N, BH;
  float scale, scale_log2;
  int causal;
};

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <int FMT>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  return FMT == 1 ? pack_bf16(a, b) : pack_f16(a, b);
}

// One work item = the 128 keys of key tile j of one (batch, head) slice.
// Items are numbered slice-group-major: (batch, head) slices in groups of
// BH_GROUP; inside a group, key tile 0 (the longest causal sweep) of every
// slice first, then key tile 1, ... CTAs take items in that order from a
// global counter, so the slices in flight at once stay few enough for their
// Q, K, V, dO and fp32 dQ rows to share L2, every SM stays busy to the end,
// and the last items are short.
struct Item {
  int bh, b, h, kv0, i0, n;
};
__device__ __forceinline__ Item decode_item(int item, const Params& p) {
  const int nkt = (p.N + BN - 1) / BN;
  const int g = item / (BH_GROUP * nkt);
  const int rem = item - g * BH_GROUP * nkt;
  const int gsz = min(BH_GROUP, p.BH - g * BH_GROUP);
  const int j = rem / gsz;
  Item it;
  it.bh = g * BH_GROUP + rem % gsz;
  it.b = it.bh / p.H;
  it.h = it.bh % p.H;
  it.kv0 = j * BN;
  it.i0 = p.causal ? (it.kv0 / BM) : 0;
  it.n = (p.N + BM - 1) / BM - it.i0;  // >= 1 since kv0 < N
  return it;
}

// Persistent: one CTA per SM. Its producer warp takes the next work item
// from p.work_counter and passes the id to the other roles through a small
// ring (item_full / item_empty); id >= n_items ends every role's loop. Every
// per-tile barrier completes once per query tile, so its phase is the
// CTA-wide running tile count g (across items), and k_full / v_full /
// k_empty / epi_staged / epi_v_free complete once per item.
template <int FMT, int HD>
__global__ void __launch_bounds__(THREADS, 1)
fa_bwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
              const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
              const __grid_constant__ CUtensorMap tdk, const __grid_constant__ CUtensorMap tdv,
              const Params p) {
  // No static shared memory is declared, so the dynamic block starts at the
  // (1 KiB-aligned) base of the CTA's window; the 128-byte swizzle needs
  // 1 KiB-aligned tiles and there is no room left for realignment padding.
  using L = Layout<HD>;
  constexpr int D = HD, KC = L::KC, TILE = L::TILE;
  constexpr int K_OFF = L::K_OFF, V_OFF = L::V_OFF, Q_OFF = L::Q_OFF, DO_OFF = L::DO_OFF;
  constexpr int DS_OFF = L::DS_OFF, STG_OFF = L::STG_OFF, STAT_OFF = L::STAT_OFF;
  constexpr int BAR_OFF = L::BAR_OFF, SLOT_OFF = L::SLOT_OFF, ITEM_OFF = L::ITEM_OFF;
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicCAS(&g_lsb_device_error, 0, 0xB00);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* k_full = bars;
  uint64_t* v_full = k_full + 1;
  uint64_t* k_empty = v_full + 1;              // the item's last dQ^T MMA (last reader of K) is done
  uint64_t* q_full = k_empty + 1;              // [NQS]
  uint64_t* q_empty = q_full + NQS;            // [NQS]
  uint64_t* stat_full = q_empty + NQS;         // [NQS]: log-sum-exp / Dsum staged
  uint64_t* do_full = stat_full + NQS;
  uint64_t* do_empty = do_full + 1;            // dV (the last reader of dO) has completed
  uint64_t* s_ready = do_empty + 1;
  uint64_t* p_ready = s_ready + 1;
  uint64_t* dp_ready = p_ready + 1;
  uint64_t* ds_ready = dp_ready + 1;
  uint64_t* dq_ready = ds_ready + 1;
  uint64_t* dq_free = dq_ready + 1;
  uint64_t* dk_done = dq_free + 1;
  // dQ staging, once per tile each: [0] warpgroup 1's 64 query rows (own
  // buffer), [1] warpgroup 2's (in the dS^T tile). red_full: staged (128
  // arrivals); red_free: the bulk reduction has read it.
  uint64_t* red_full = dk_done + 1;            // [2]
  uint64_t* red_free = red_full + 2;           // [2]
  float* stats = reinterpret_cast<float*>(smem + STAT_OFF);  // [NQS][lse2 BM | dsum BM]
  // Item epilogue: the warpgroups stage dK in the V buffer and dV in the Q
  // stage of the item's last tile as bf16 tiles (epi_staged, 256
  // arrivals); the reducer stores both with TMA ahead of the item's last dQ
  // reduction. epi_v_free (once per item) and epi_q_free[stage] (once per
  // staging in that stage) tell the producer that a buffer has been read;
  // the next item's first dP^T waits for V, its second S^T for the Q stage.
  uint64_t* epi_staged = red_free + 2;
  uint64_t* epi_v_free = epi_staged + 1;
  // The producer has issued the next item's V and dO loads (once per item;
  // after the CTA's last item, with nothing to load): the reducer issues
  // the last tile's dQ reductions only then, since the TMA unit serves its
  // bulk operations in order and the loads would otherwise wait for 64 KiB
  // of reduction traffic.
  uint64_t* vdo_issued = epi_v_free + 1;
  uint64_t* epi_q_free = vdo_issued + 1;       // [NQS]
  uint64_t* item_full = epi_q_free + NQS;      // [NIS]
  uint64_t* item_empty = item_full + NIS;      // [NIS]: 10 arrivals (MMA, reducer, 8 warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + SLOT_OFF);
  volatile int* item_ids = reinterpret_cast<volatile int*>(smem + ITEM_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = p.BH * ((p.N + BN - 1) / BN);
  // Consumer side of the work-item ring: id of the k-th item (>= n_items:
  // no more work), or -1 when the wait gave up.
  auto next_item = [&](int k, bool arrive) -> int {
    const int slot = k % NIS;
    if (!mbar_wait(&item_full[slot], (k / NIS) & 1, 0x50A)) return -1;
    const int id = item_ids[slot];
    if (arrive) mbar_arrive(&item_empty[slot]);
    return id;
  };

  if (threadIdx.x == 0) {
    mbar_init(k_full, 1);
    mbar_init(v_full, 1);
    mbar_init(k_empty, 1);
    for (int s = 0; s < NQS; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
      mbar_init(&stat_full[s], 32);
    }
    mbar_init(do_full, 1);
    mbar_init(do_empty, 1);
    mbar_init(s_ready, 1);
    mbar_init(p_ready, 256);
    mbar_init(dp_ready, 1);
    mbar_init(ds_ready, 256);
    mbar_init(dq_ready, 1);
    mbar_init(dq_free, 256);
    mbar_init(dk_done, 1);
    for (int i = 0; i < 2; ++i) { mbar_init(&red_full[i], 128); mbar_init(&red_free[i], 1); }
    mbar_init(epi_staged, 256);
    mbar_init(epi_v_free, 1);
    mbar_init(vdo_issued, 1);
    for (int i = 0; i < NQS; ++i) mbar_init(&epi_q_free[i], 1);
    for (int i = 0; i < NIS; ++i) { mbar_init(&item_full[i], 1); mbar_init(&item_empty[i], 10); }
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

  uint8_t* sK = smem + K_OFF;
  uint8_t* sV = smem + V_OFF;
  uint8_t* sQ = smem + Q_OFF;
  uint8_t* sDO = smem + DO_OFF;
  uint8_t* sDS = smem + DS_OFF;
  uint8_t* sSTG = smem + STG_OFF;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    reg_dealloc<112>();
    if (lane == 0) {
      prefetch_tmap(&tq); prefetch_tmap(&tk); prefetch_tmap(&tv); prefetch_tmap(&tdo);
      prefetch_tmap(&tdk); prefetch_tmap(&tdv);
    }
    int g = 0;  // running query-tile count of this CTA
    bool ok = true;
    // Claims work item k: takes the next id from the global counter and
    // publishes it in ring slot k % NIS (once item k - NIS has been taken
    // by every role). The id of item k+1 is claimed while item k's last
    // query tile loads, and its K / V tiles are prefetched into L2 then, so
    // the K / V loads at the item boundary read L2 instead of HBM.
    auto claim = [&](int k) -> int {
      const int slot = k % NIS;
      if (k >= NIS && !mbar_wait_warp(&item_empty[slot], ((k / NIS) - 1) & 1, 0x504)) return -1;
      int id = 0;
      if (lane == 0) {
        id = atomicAdd(p.work_counter, 1);
        item_ids[slot] = id;
        mbar_arrive(&item_full[slot]);  // release: the id is visible to its waiters
        if (id < n_items) {
          const Item nw = decode_item(id, p);
          for (int kc = 0; kc < KC; ++kc) {
            tma_prefetch_l2_4d(&tk, kc * 64, nw.kv0, nw.h, nw.b);
            tma_prefetch_l2_4d(&tv, kc * 64, nw.kv0, nw.h, nw.b);
          }
        }
      }
      return __shfl_sync(0xffffffffu, id, 0);
    };
    uint32_t q_pend = 0, q_phase = 0;  // per Q stage: dV staging pending / its phase
    int item = claim(0);
    for (int k = 0; ok && item >= 0 && item < n_items; ++k) {
      const Item w = decode_item(item, p);
      const float* lse_bh = p.lse + (int64_t)w.bh * p.N;
      const float* dsum_bh = p.dsum + (int64_t)w.bh * p.N;
      int next = -1;
      for (int it = 0; it < w.n; ++it, ++g) {
        const int s = g % NQS;
        // Stage s is reused once the MMAs of tile g-NQS (and so every read of
        // its statistics, which precede ds_ready) have completed.
        if (g >= NQS && !mbar_wait_warp(&q_empty[s], ((g / NQS) - 1) & 1, 0x501)) { ok = false; break; }
        // Tile g-NQS ended an item: its dV staging in this stage must have
        // been stored first.
        if ((q_pend >> s) & 1) {
          if (!mbar_wait_warp(&epi_q_free[s], (q_phase >> s) & 1, 0x506)) { ok = false; break; }
          q_phase ^= 1u << s;
          q_pend &= ~(1u << s);
        }
        const int m0 = (w.i0 + it) * BM;
        if (lane == 0) {
          mbar_arrive_expect_tx(&q_full[s], TILE);
          for (int kc = 0; kc < KC; ++kc)
            tma_load_4d(sQ + s * TILE + kc * CHUNK, &tq, &q_full[s], kc * 64, m0, w.h, w.b);
        }
        // Per-query statistics of this tile: log2-scaled LSE and Dsum.
        float* st = stats + s * 2 * BM;
#pragma unroll
        for (int u = 0; u < BM / 32; ++u) {
          const int c = lane + 32 * u;
          const bool in = m0 + c < p.N;
          st[c] = in ? __ldg(lse_bh + m0 + c) * 1.4426950408889634f : 0.f;
          st[BM + c] = in ? __ldg(dsum_bh + m0 + c) : 0.f;
        }
        mbar_arrive(&stat_full[s]);
        // K of this item replaces the previous item's once its last dQ^T
        // (the last reader of K) has completed.
        if (it == 0) {
          if (k > 0 && !mbar_wait_warp(k_empty, (k - 1) & 1, 0x507)) { ok = false; break; }
          if (lane == 0) {
            mbar_arrive_expect_tx(k_full, TILE);
            for (int kc = 0; kc < KC; ++kc)
              tma_load_4d(sK + kc * CHUNK, &tk, k_full, kc * 64, w.kv0, w.h, w.b);
          }
        }
        // V replaces the previous item's dK staging once its TMA store has
        // read it (which follows every MMA of that item); dO(g) replaces
        // dO(g-1) once dV(g-1) has read it.
        if (it == 0 && k > 0 && !mbar_wait_warp(epi_v_free, (k - 1) & 1, 0x503)) { ok = false; break; }
        if (g > 0 && !mbar_wait_warp(do_empty, (g - 1) & 1, 0x502)) { ok = false; break; }
        if (lane == 0) {
          if (it == 0) {
            mbar_arrive_expect_tx(v_full, TILE);
            for (int kc = 0; kc < KC; ++kc)
              tma_load_4d(sV + kc * CHUNK, &tv, v_full, kc * 64, w.kv0, w.h, w.b);
          }
          mbar_arrive_expect_tx(do_full, TILE);
          for (int kc = 0; kc < KC; ++kc)
            tma_load_4d(sDO + kc * CHUNK, &tdo, do_full, kc * 64, m0, w.h, w.b);
          if (it == 0 && k > 0) mbar_arrive(vdo_issued);
        }
        if (it == w.n - 1) {
          q_pend |= 1u << s;
          next = claim(k + 1);
        }
      }
      item = next;
    }
    if (ok && item >= n_items && lane == 0) mbar_arrive(vdo_issued);  // for the CTA's last item
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issue --
    reg_dealloc<112>();
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_f16(128, BM, FMT, 0, 0);   // K-major A and B
      constexpr uint32_t ID_ACC = idesc_f16(128, D, FMT, 0, 1);  // TS; B (dO, Q) MN-major
      // A (K^T), B (dS^T) MN-major. M stays 128 when D = 64: A's second
      // 64-row group is then read from the V tile after K, and the TMEM
      // lanes 64-127 it produces are never read.
      constexpr uint32_t ID_DQ = idesc_f16(128, BM, FMT, 1, 1);
      const uint32_t k_base = smem_u32(sK), v_base = smem_u32(sV);
      const uint32_t q_base = smem_u32(sQ), do_base = smem_u32(sDO), ds_base = smem_u32(sDS);
      // X^T = A B^T with A the [128][D] K or V tile, B the [BM][D] Q or dO tile.
      auto issue_t = [&](uint32_t d_col, uint32_t a_base, uint32_t b_base) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t a = smem_desc_sw128(a_base + (kk / 4) * CHUNK + (kk % 4) * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(b_base + (kk / 4) * CHUNK + (kk % 4) * 32, 16, 1024);
          mma_ss(tmem + d_col, a, bd, ID_S, kk > 0);
        }
      };
      // Acc[128 keys][D] += A_tmem[128][BM q] * B[BM q][D]  (B MN-major, rows = q).
      // Warpgroup g packed the 16-bit values of its query columns [64g, 64g+64)
      // into TMEM columns T_S + 64g + a_off + [0, 32): K-step kk (queries
      // [16kk, 16kk+16)) reads 8 columns there.
      auto issue_acc = [&](uint32_t d_col, uint32_t a_off, uint32_t b_base, bool acc) {
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk) {
          const uint64_t bd = smem_desc_sw128(b_base + kk * 2048, CHUNK, 1024);
          mma_ts(tmem + d_col, tmem + T_S + (kk >> 2) * 64 + a_off + (kk & 3) * 8, bd, ID_ACC,
                 (acc || kk > 0) ? 1u : 0u);
        }
      };
      // S^T(g) and dP^T(g). dP^T overwrites dQ^T(g-1) once the warpgroups
      // have loaded it (dq_free).
      // An item's first tile also waits for its K (before S^T) and V (before
      // dP^T).
      auto issue_s_dp = [&](int gg, int k, bool first) -> bool {
        const int s = gg % NQS;
        if (first && !mbar_wait(k_full, k & 1, 0x601)) return false;
        if (!mbar_wait(&q_full[s], (gg / NQS) & 1, 0x605)) return false;
        tc_fence_after();
        issue_t(T_S, k_base, q_base + s * TILE);
        mma_commit(s_ready);
        if ((gg > 0 && !mbar_wait(dq_free, (gg - 1) & 1, 0x606)) ||
            !mbar_wait(do_full, gg & 1, 0x608) || (first && !mbar_wait(v_full, k & 1, 0x609)))
          return false;
        tc_fence_after();
        issue_t(T_DP, v_base, do_base);
        mma_commit(dp_ready);
        return true;
      };
      int g = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int item = next_item(k, true);
        if (item < 0 || item >= n_items) break;
        const Item w = decode_item(item, p);
        if (!issue_s_dp(g, k, true)) { ok = false; break; }
        for (int it = 0; it < w.n; ++it, ++g) {
          const int s = g % NQS;
          const uint32_t ph = g & 1;
          // dV(0) of an item overwrites the previous item's dV: the
          // warpgroups read it out (epilogue) before their p_ready.
          if (!mbar_wait(p_ready, ph, 0x603)) { ok = false; break; }
          tc_fence_after();
          issue_acc(T_DV, 0, do_base, it > 0);
          mma_commit(do_empty);
          if (!mbar_wait(ds_ready, ph, 0x604)) { ok = false; break; }
          tc_fence_after();
          // dQ^T(g) = K^T dS^T over the 128 keys, into the dP^T columns
          // (every read of dP^T(g) preceded ds_ready).
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t a = smem_desc_sw128(k_base + kk * 2048, CHUNK, 1024);
            const uint64_t bd = smem_desc_sw128(ds_base + kk * 2048, CHUNK, 1024);
            mma_ss(tmem + T_DP, a, bd, ID_DQ, kk > 0);
          }
          mma_commit(dq_ready);
          if (it + 1 == w.n) mma_commit(k_empty);  // the item's last read of K
          issue_acc(T_DK, 32, q_base + s * TILE, it > 0);
          mma_commit(dk_done);
          mma_commit(&q_empty[s]);
          // tcgen05.mma instructions of one thread execute in issue order, so
          // S^T(g+1) overwrites P^T / dS^T(g) only after dV(g) and dK(g)
          // have read them.
          if (it + 1 < w.n && !issue_s_dp(g + 1, k, false)) { ok = false; break; }
        }
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------- dQ reducer --
    // Adds each staged 64-row dQ half-tile into the fp32 dQ buffer (rows are
    // contiguous there) with one bulk reduction per half; the dS^T-tile half
    // goes first, since the next dS^T write waits for it to be read. An
    // item's last tile first hands the item's staged dK and dV tiles to TMA
    // stores, whose buffers are released once read, and lets the next
    // item's V / dO loads go ahead of its reductions (vdo_issued).
    reg_dealloc<112>();
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int kk = 0; ok; ++kk) {
        const int item = next_item(kk, true);
        if (item < 0 || item >= n_items) break;
        const Item w = decode_item(item, p);
        for (int it = 0; it < w.n; ++it, ++g) {
          const uint32_t ph = g & 1;
          const int64_t m0 = (int64_t)(w.i0 + it) * BM;
          const bool last = it + 1 == w.n;
          if (last) {
            // dK store, V buffer released, next V / dO loads issued, then the
            // dV store and this tile's reductions (every earlier bulk group
            // has been read by now).
            ok = mbar_wait(epi_staged, kk & 1, 0x902);
            if (!ok) break;
            for (int kc = 0; kc < KC; ++kc)
              tma_store_4d(&tdk, sV + kc * CHUNK, kc * 64, w.kv0, w.h, w.b);
            bulk_commit();
            bulk_wait_read();
            mbar_arrive(epi_v_free);
            ok = mbar_wait(vdo_issued, kk & 1, 0x903);
            if (!ok) break;
            for (int kc = 0; kc < KC; ++kc)
              tma_store_4d(&tdv, sQ + (g % NQS) * TILE + kc * CHUNK, kc * 64, w.kv0, w.h, w.b);
            bulk_commit();
          }
          for (int k = 1; k >= 0 && ok; --k) {
            ok = mbar_wait(&red_full[k], ph, 0x901);
            const int rows = (int)min((int64_t)STAGE_ROWS, p.N - (m0 + k * STAGE_ROWS));
            if (ok && rows > 0)
              bulk_reduce_add_f32(p.dq_acc + ((int64_t)w.bh * p.N + m0 + k * STAGE_ROWS) * D,
                                  reinterpret_cast<const float*>(k ? sDS : sSTG), rows * D * 4);
            bulk_commit();  // an empty group when nothing was issued
          }
          if (!ok) break;
          if (last) {
            bulk_wait_read_2();
            mbar_arrive(&epi_q_free[g % NQS]);
          }
          bulk_wait_read_1();
          mbar_arrive(&red_free[1]);
          bulk_wait_read();
          mbar_arrive(&red_free[0]);
        }
      }
      bulk_wait_all();  // every store and reduction has landed before the CTA exits
    }
  } else if (warp < 4) {
    reg_dealloc<112>();
  } else {
    // ------------------------------------------------------------------------
    // Two warpgroups split the 128 query columns of each tile (64 each):
    // thread = key (TMEM lane) for P^T / dS^T, then thread = head-dim index
    // for its 64 dQ^T columns. Item epilogue: warpgroup 1 writes dV,
    // warpgroup 2 dK, while the next item's K / V load and first S^T run.
    reg_alloc<176>();
    const int half = warp >> 3;                  // 0: q cols [0,64), 1: [64,128)
    const int r = (threadIdx.x & 127);           // TMEM lane: key, then head-dim index
    const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const float sl2 = p.scale_log2;
    const int cb = half * 64;                    // first query column of this half
    const uint32_t my_s = lane_addr + T_S + cb;  // this half's S^T columns
    int g = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      int item = 0;
      if (lane == 0) item = next_item(k, true);
      item = __shfl_sync(0xffffffffu, item, 0);
      if (item < 0 || item >= n_items) break;
      const Item w = decode_item(item, p);
      const int key = w.kv0 + r;
      const int qlo = p.causal ? key : 0;  // first valid q for this key
      for (int it = 0; it < w.n; ++it, ++g) {
        const uint32_t ph = g & 1;
        const int m0 = (w.i0 + it) * BM;
        const float* st = stats + (g % NQS) * 2 * BM;
        if (!mbar_wait_warp(&stat_full[g % NQS], (g / NQS) & 1, 0x705)) { ok = false; break; }
        if (!mbar_wait_warp(s_ready, ph, 0x701)) { ok = false; break; }
        tc_fence_after();
        uint32_t sv[64];
        tmem_ld32(my_s, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_ld32(my_s + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        tmem_ld_wait();
        // Masks: causal (q < key), and rows/columns past the sequence end.
        const bool need_mask =
            (m0 + BM > p.N) || (w.kv0 + BN > p.N) || (p.causal && m0 < w.kv0 + BN);
        float pf[64];
        uint32_t pk[32];
        // The mask test is hoisted out of the exp2 loop: a branch per element
        // pair would cut the loop into blocks too small to hide MUFU latency.
#pragma unroll
        for (int cc = 0; cc < 32; ++cc) {
          const float2 l2 = *reinterpret_cast<const float2*>(st + cb + 2 * cc);  // shared broadcast
          pf[2 * cc] = ex2(fmaf(__uint_as_float(sv[2 * cc]), sl2, -l2.x));
          pf[2 * cc + 1] = ex2(fmaf(__uint_as_float(sv[2 * cc + 1]), sl2, -l2.y));
        }
        if (need_mask) {
          const int qhi = min(p.N - (m0 + cb), 64);  // columns c < qhi are real queries
          const int clo = key >= p.N ? 64 : qlo - (m0 + cb);  // columns c < clo are masked
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c < clo || c >= qhi) pf[c] = 0.f;
        }
#pragma unroll
        for (int cc = 0; cc < 32; ++cc) pk[cc] = pack2<FMT>(pf[2 * cc], pf[2 * cc + 1]);
        // P^T into the first 32 columns of this half's own S^T range (the
        // other warpgroup's unread scores are never overwritten).
        tmem_st32(my_s, pk);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(p_ready);

        if (!mbar_wait_warp(dp_ready, ph, 0x702)) { ok = false; break; }
        tc_fence_after();
        tmem_ld32(lane_addr + T_DP + cb, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_ld32(lane_addr + T_DP + cb + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        tmem_ld_wait();
#pragma unroll
        for (int cc = 0; cc < 32; ++cc) {
          const float2 ds2 = *reinterpret_cast<const float2*>(st + BM + cb + 2 * cc);
          pk[cc] = pack2<FMT>(pf[2 * cc] * (__uint_as_float(sv[2 * cc]) - ds2.x),
                              pf[2 * cc + 1] * (__uint_as_float(sv[2 * cc + 1]) - ds2.y));
        }
        tmem_st32(my_s + 32, pk);  // dS^T beside P^T
        // dS^T row -> shared chunk `half` (128-byte swizzle) for the dQ^T GEMM,
        // once the bulk reduction has read the previous tile's second dQ
        // staging half from the same buffer.
        if (g > 0 && !mbar_wait_warp(&red_free[1], (g - 1) & 1, 0x703)) { ok = false; break; }
        {
          uint8_t* rowp = sDS + half * CHUNK + r * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(rowp + ((c ^ (r & 7)) << 4)) =
                make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        }
        fence_proxy_async_smem();
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(ds_ready);

        // dQ^T(g), thread = head-dim index r, this half's 64 query columns.
        if (!mbar_wait_warp(dq_ready, ph, 0x704)) { ok = false; break; }
        tc_fence_after();
        tmem_ld32(lane_addr + T_DP + cb, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_ld32(lane_addr + T_DP + cb + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(dq_free);
        // Warpgroup 1 reuses its buffer once the previous tile's rows have been
        // read; warpgroup 2's half of the dS^T tile is free (dQ^T(g) is done).
        if (half == 0 && g > 0 && !mbar_wait_warp(&red_free[0], (g - 1) & 1, 0x706)) {
          ok = false;
          break;
        }
        float* stage = reinterpret_cast<float*>(half == 0 ? sSTG : sDS);
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (D == 128 || r < D) stage[c * D + r] = __uint_as_float(sv[c]) * p.scale;
        fence_proxy_async_smem();
        mbar_arrive(&red_full[half]);
      }
      if (!ok) break;
      // Item epilogue: warpgroup 1 stages this key's dV row (in the last
      // tile's Q stage), warpgroup 2 its dK row (in the V buffer); dk_done:
      // every MMA of the item, so also the last readers of Q and V, has
      // completed. The next item's dV(0) / dK(0) overwrite
      // these columns only after this warpgroup's p_ready of that tile.
      if (!mbar_wait_warp(dk_done, (g - 1) & 1, 0x707)) { ok = false; break; }
      tc_fence_after();
      // Staged as bf16 in the TMA store layout ([2 chunks][128 keys][64 d],
      // 128-byte swizzle); the store skips keys past the sequence end.
      const uint32_t col = half == 0 ? T_DV : T_DK;
      const float mul = half == 0 ? 1.f : p.scale;
      uint8_t* rowp0 = (half == 0 ? sQ + ((g - 1) % NQS) * TILE : sV) + r * 128;
#pragma unroll
      for (int i = 0; i < D / 32; ++i) {
        uint32_t v[32];
        tmem_ld32(lane_addr + col + 32 * i, v);
        tmem_ld_wait();
        uint32_t pk2[16];
#pragma unroll
        for (int cc = 0; cc < 16; ++cc)
          pk2[cc] = pack2<FMT>(__uint_as_float(v[2 * cc]) * mul, __uint_as_float(v[2 * cc + 1]) * mul);
        uint8_t* rowp = rowp0 + (i >> 1) * CHUNK;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int unit = (i & 1) * 4 + j;  // 16-byte unit inside the 128-byte row segment
          *reinterpret_cast<uint4*>(rowp + ((unit ^ (r & 7)) << 4)) =
              make_uint4(pk2[4 * j], pk2[4 * j + 1], pk2[4 * j + 2], pk2[4 * j + 3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(epi_staged);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace fa_bwd


bool attn_bwd_tc_eligible(const void* q, const void* k, const void* v, const void* o,
                          const void* dout, const void* dq, const void* dk, const void* dv,
                          int64_t B, int64_t H, int64_t N, int64_t D, const int64_t* sq,
                          const int64_t* sk, const int64_t* sv, const int64_t* so,
                          const int64_t* sdo, const int64_t* sdq, const int64_t* sdk,
                          const int64_t* sdv, int dtype) {
  (void)o; (void)so; (void)dq; (void)sdq;
  if (dtype != LSB_DTYPE_BF16 && dtype != LSB_DTYPE_F16) return false;
  if (D != 64 && D != 128) return false;
  if (N >= (1LL << 30) || B * H * ((N + fa_bwd::BN - 1) / fa_bwd::BN) > 0x7fffffff) return false;
  if (!tma_ok(q, B, H, N, sq, 2) || !tma_ok(k, B, H, N, sk, 2) || !tma_ok(v, B, H, N, sv, 2) ||
      !tma_ok(dout, B, H, N, sdo, 2))
    return false;
  // dK and dV are written with TMA stores.
  return tma_ok(dk, B, H, N, sdk, 2) && tma_ok(dv, B, H, N, sdv, 2);
}

template <int FMT, int HD>
static int launch_fa_bwd(const void* q, const void* k, const void* v, const void* dout,
                         const float* lse, void* dk, void* dv, int64_t B, int64_t H, int64_t N,
                         const int64_t* sq, const int64_t* sk, const int64_t* sv,
                         const int64_t* sdo, const int64_t* sdk, const int64_t* sdv, float scale,
                         int causal, int dtype, const float* dsum, float* dq_acc,
                         int* work_counter, cudaStream_t st) {
  using namespace fa_bwd;
  constexpr int D = HD;
  constexpr int SMEM = Layout<HD>::SMEM;
  CUtensorMap mq, mk, mv, mdo, mdk, mdv;
  int rc = make_bhnd_map(&mq, q, dtype, B, H, N, D, sq, 64, BM);
  if (!rc) rc = make_bhnd_map(&mdo, dout, dtype, B, H, N, D, sdo, 64, BM);
  if (!rc) rc = make_bhnd_map(&mk, k, dtype, B, H, N, D, sk, 64, BN);
  if (!rc) rc = make_bhnd_map(&mv, v, dtype, B, H, N, D, sv, 64, BN);
  if (!rc) rc = make_bhnd_map(&mdk, dk, dtype, B, H, N, D, sdk, 64, BN);
  if (!rc) rc = make_bhnd_map(&mdv, dv, dtype, B, H, N, D, sdv, 64, BN);
  if (rc) return rc;
  Params p;
  p.lse = lse; p.dsum = dsum; p.dq_acc = dq_acc;
  p.work_counter = work_counter;
  p.H = (int)H; p.N = (int)N; p.BH = (int)(B * H);
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  auto kern = fa_bwd_kernel<FMT, HD>;
  static SmemLimit smem_limit;
  if (int rc_ = smem_limit.ensure(kern, SMEM, "attn_bwd_tc smem attribute")) return rc_;
  // Persistent: one CTA per SM (shared memory and TMEM allow no more).
  const int64_t n_items = B * H * ((N + BN - 1) / BN);
  dim3 grid((unsigned)std::min<int64_t>(n_items, num_sms()));
  kern<<<grid, THREADS, SMEM, st>>>(mq, mk, mv, mdo, mdk, mdv, p);
  LSB_CHECK_LAUNCH("attn_bwd_tc");
  return LSB_OK;
}

int attn_bwd_tc(const void* q, const void* k, const void* v, const void* o, const void* dout,
                const float* lse, void* dq, void* dk, void* dv, int64_t B, int64_t H, int64_t N,
                int64_t D, const int64_t* sq, const int64_t* sk, const int64_t* sv,
                const int64_t* so, const int64_t* sdo, const int64_t* sdq, const int64_t* sdk,
                const int64_t* sdv, float scale, int causal, int dtype, float* dsum,
                float* dq_acc, cudaStream_t st) {
  auto S4 = [](const int64_t* s) { return Strides4{s[0], s[1], s[2], s[3]}; };
  const bool bf = dtype == LSB_DTYPE_BF16;
  // The work-item counter sits in the 256 bytes after the (256-byte padded)
  // dQ accumulator (lsb_attn_bwd_workspace_size). The Dsum pass zeroes both
  // in the same launch (else one memset does).
  int* work_counter = reinterpret_cast<int*>(reinterpret_cast<char*>(dq_acc) + align256(4 * B * H * N * D));
  bool zeroed = false;
  int rc = bf ? launch_dsum<__nv_bfloat16>(o, dout, dsum, B, H, N, D, S4(so), S4(sdo), st, dq_acc,
                                           work_counter, &zeroed)
              : launch_dsum<__half>(o, dout, dsum, B, H, N, D, S4(so), S4(sdo), st, dq_acc,
                                    work_counter, &zeroed);
  if (rc) return rc;
  if (!zeroed)
    LSB_CUDA_OK(cudaMemsetAsync(dq_acc, 0, (size_t)align256(4 * B * H * N * D) + sizeof(int), st),
                "attn_bwd dQ accumulator memset");
  auto fa = bf ? (D == 128 ? launch_fa_bwd<1, 128> : launch_fa_bwd<1, 64>)
               : (D == 128 ? launch_fa_bwd<0, 128> : launch_fa_bwd<0, 64>);
  rc = fa(q, k, v, dout, lse, dk, dv, B, H, N, sq, sk, sv, sdo, sdk, sdv, scale, causal, dtype, dsum,
          dq_acc, work_counter, st);
  if (rc) return rc;
  return bf ? launch_dq_cast<__nv_bfloat16>(dq_acc, dq, B, H, N, D, S4(sdq), st)
            : launch_dq_cast<__half>(dq_acc, dq, B, H, N, D, S4(sdq), st);
}


int attn_bwd_tc_device_error(bool reset) {
  return sm100::tu_device_error(reset);
}

}  // namespace lsb
