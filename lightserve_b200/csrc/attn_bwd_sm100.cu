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
// tiles of 64 rows (causal: starting at the diagonal). Everything is computed
// transposed so the 128 keys are the TMEM lanes:
//   S^T  = K Q^T      (SS MMA)  -> TMEM cols [0,64)
//   dP^T = V dO^T     (SS MMA)  -> TMEM cols [64,128)
//   dV  += P^T dO     (TS MMA, P^T packed to 16 bits over S^T)  -> [128,256)
//   dK  += dS^T Q     (TS MMA, dS^T packed over dP^T)           -> [256,384)
//   dQ^T = K^T dS^T   (SS MMA, K^T read MN-major from the K tile, dS^T
//                      from a 128-byte-swizzled shared tile)    -> [384,448)
// Warp 0 streams K/V once and Q/dO tiles (plus each tile's log-sum-exp and
// Dsum) through a 2-stage ring; warp 1 owns TMEM and issues the MMAs; warp 2
// adds each finished 64-row dQ tile into the fp32 dQ buffer with one bulk
// shared->global reduction (double-buffered staging). Warpgroups 1 and 2 split
// every tile's 64 query columns: thread = key for P^T / dS^T, thread =
// head-dim index when staging dQ^T; the previous tile's dQ^T is staged while
// the current dP^T completes.
// All mbarrier waits are bounded (sm100.cuh).
#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace lsb {

struct Strides4 {
  int64_t b, h, n, d;
};
template <typename T>
int launch_dsum(const void* o, const void* dout, float* dsum, int64_t B, int64_t H, int64_t N,
                int64_t D, Strides4 so, Strides4 sdo, cudaStream_t st);
template <typename T>
int launch_dq_cast(const float* dq_acc, void* dq, int64_t B, int64_t H, int64_t N, int64_t D,
                   Strides4 sdq, cudaStream_t st);

namespace fa_bwd {

using namespace sm100;

constexpr int BN = 128;   // keys per CTA (TMEM lanes)
constexpr int BM = 64;    // query rows per inner tile
constexpr int D = 128;    // head dim served by this kernel
constexpr int THREADS = 384;
constexpr int KV_CHUNK = 128 * 128;  // [128 rows][64 cols] 16-bit box
constexpr int Q_CHUNK = 64 * 128;    // [64 rows][64 cols] 16-bit box
constexpr int KC = D / 64;

constexpr int K_OFF = 0;
constexpr int V_OFF = K_OFF + KC * KV_CHUNK;
constexpr int NQS = 3;    // Q / dO / statistics ring stages
constexpr int Q_OFF = V_OFF + KC * KV_CHUNK;          // [NQS][KC] Q chunks
constexpr int DO_OFF = Q_OFF + NQS * KC * Q_CHUNK;    // [NQS][KC] dO chunks
constexpr int DS_OFF = DO_OFF + NQS * KC * Q_CHUNK;   // dS^T [2][128 keys][64 q] swizzled
constexpr int DS_BYTES = BN * BM * 2;
constexpr int RED_OFF = DS_OFF + 2 * DS_BYTES;        // dQ staging [64 q][D] fp32
constexpr int STAT_OFF = RED_OFF + BM * D * 4;        // [NQS][2][64] floats: lse2, dsum
constexpr int BAR_OFF = STAT_OFF + NQS * 2 * BM * 4;
// kv_full, q_full[NQS], q_empty[NQS], s_ready[2], dp_ready, p_ready[2], ds_ready,
// dv_done, dk_done, dq_ready, dq_free, stat_full[NQS], red_full, red_free
constexpr int NBAR = 1 + 3 * NQS + 2 + 1 + 2 + 7;
constexpr int SLOT_OFF = BAR_OFF + NBAR * 8;
constexpr int SMEM = SLOT_OFF + 16 + 1024;
static_assert(SMEM <= 232448, "backward tile set exceeds the 227 KiB shared-memory limit");

// TMEM columns: S^T double-buffered (tile it uses T_S + (it & 1) * 64).
constexpr uint32_t T_S = 0, T_DP = 128, T_DV = 192, T_DK = 320, T_DQ = 448;

struct Params {
  const float* lse;
  const float* dsum;
  float* dq_acc;
  void* dk;
  void* dv;
  int64_t sdk_b, sdk_h, sdk_n, sdv_b, sdv_h, sdv_n;
  int H, N;
  float scale, scale_log2;
  int causal;
};

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void named_bar(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

#ifdef LSB_BWD_TRACE
// Debug-build timeline of CTA (0, 0): clock64 per event and query tile.
__device__ long long g_bwd_trace[16][64];
#define BWD_TRACE(cond, ev, it)                                               \
  do {                                                                        \
    if ((cond) && blockIdx.x == 0 && blockIdx.y == 0 && (it) < 64)            \
      g_bwd_trace[ev][it] = clock64();                                        \
  } while (0)
#else
#define BWD_TRACE(cond, ev, it) \
  do {                          \
  } while (0)
#endif

template <int FMT>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  return FMT == 1 ? pack_bf16(a, b) : pack_f16(a, b);
}

template <int FMT>
__global__ void __launch_bounds__(THREADS, 1)
fa_bwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
              const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
              const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;                 // [NQS]
  uint64_t* q_empty = q_full + NQS;            // [NQS]
  uint64_t* s_ready = q_empty + NQS;           // [2]: per S^T buffer
  uint64_t* dp_ready = s_ready + 2;
  uint64_t* p_ready = dp_ready + 1;            // [2]: per S^T buffer
  uint64_t* ds_ready = p_ready + 2;
  uint64_t* dv_done = ds_ready + 1;
  uint64_t* dk_done = dv_done + 1;
  uint64_t* dq_ready = dk_done + 1;
  uint64_t* dq_free = dq_ready + 1;
  uint64_t* stat_full = dq_free + 1;           // [NQS]: log-sum-exp / Dsum staged
  uint64_t* red_full = stat_full + NQS;        // dQ tile staged (256 arrivals)
  uint64_t* red_free = red_full + 1;           // its bulk reduction has read it
  float* stats = reinterpret_cast<float*>(smem + STAT_OFF);  // [NQS][lse2 64 | dsum 64]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + SLOT_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.x;  // key tile (ascending = most query tiles first when causal)
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int kv0 = j * BN;
  const int nq_all = (p.N + BM - 1) / BM;
  const int i0 = p.causal ? (kv0 / BM) : 0;
  const int n = nq_all - i0;  // >= 1 since kv0 < N

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < NQS; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
      mbar_init(&stat_full[s], 32);
    }
    for (int i = 0; i < 2; ++i) { mbar_init(&s_ready[i], 1); mbar_init(&p_ready[i], 256); }
    mbar_init(dp_ready, 1);
    mbar_init(ds_ready, 256);
    mbar_init(dv_done, 1);
    mbar_init(dk_done, 1);
    mbar_init(dq_ready, 1);
    mbar_init(dq_free, 256);
    mbar_init(red_full, 256);
    mbar_init(red_free, 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    reg_dealloc<72>();
    const float* lse_bh = p.lse + (int64_t)bh * p.N;
    const float* dsum_bh = p.dsum + (int64_t)bh * p.N;
    if (lane == 0) {
      prefetch_tmap(&tq); prefetch_tmap(&tk); prefetch_tmap(&tv); prefetch_tmap(&tdo);
      mbar_arrive_expect_tx(kv_full, 2 * KC * KV_CHUNK);
      for (int kc = 0; kc < KC; ++kc) {
        tma_load_4d(sK + kc * KV_CHUNK, &tk, kv_full, kc * 64, kv0, h, b);
        tma_load_4d(sV + kc * KV_CHUNK, &tv, kv_full, kc * 64, kv0, h, b);
      }
    }
    for (int it = 0; it < n; ++it) {
      const int s = it % NQS;
      // Stage s is reused once the MMAs of tile it-NQS (and so every read of
      // its statistics, which precede ds_ready) have completed.
      if (it >= NQS && !mbar_wait_warp(&q_empty[s], ((it / NQS) - 1) & 1, 0x501)) break;
      const int m0 = (i0 + it) * BM;
      if (lane == 0) {
        mbar_arrive_expect_tx(&q_full[s], 2 * KC * Q_CHUNK);
        for (int kc = 0; kc < KC; ++kc) {
          tma_load_4d(sQ + (s * KC + kc) * Q_CHUNK, &tq, &q_full[s], kc * 64, m0, h, b);
          tma_load_4d(sDO + (s * KC + kc) * Q_CHUNK, &tdo, &q_full[s], kc * 64, m0, h, b);
        }
      }
      // Per-query statistics of this tile: log2-scaled LSE and Dsum.
      float* st = stats + s * 2 * BM;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int c = lane + 32 * u;
        const bool in = m0 + c < p.N;
        st[c] = in ? __ldg(lse_bh + m0 + c) * 1.4426950408889634f : 0.f;
        st[BM + c] = in ? __ldg(dsum_bh + m0 + c) : 0.f;
      }
      mbar_arrive(&stat_full[s]);
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issue --
    reg_dealloc<72>();
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_f16(128, BM, FMT, 0, 0);   // K-major A and B
      constexpr uint32_t ID_DV = idesc_f16(128, D, FMT, 0, 1);   // B (dO, Q) MN-major
      constexpr uint32_t ID_DQ = idesc_f16(128, BM, FMT, 1, 1);  // A (K^T), B (dS^T) MN-major
      const uint32_t k_base = smem_u32(sK), v_base = smem_u32(sV);
      const uint32_t q_base = smem_u32(sQ), do_base = smem_u32(sDO), ds_base = smem_u32(sDS);
      // X^T = A B^T with A the [128][D] K or V tile, B the [64][D] Q or dO tile.
      auto issue_t = [&](uint32_t d_col, uint32_t a_base, uint32_t b_base) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t a = smem_desc_sw128(a_base + (kk / 4) * KV_CHUNK + (kk % 4) * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(b_base + (kk / 4) * Q_CHUNK + (kk % 4) * 32, 16, 1024);
          mma_ss(tmem + d_col, a, bd, ID_S, kk > 0);
        }
      };
      // Acc[128 keys][D] += A_tmem[128][64 q] * B[64 q][D]  (B MN-major, rows = q)
      auto issue_acc = [&](uint32_t d_col, uint32_t a_col, uint32_t b_base, bool acc) {
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk) {
          const uint64_t bd = smem_desc_sw128(b_base + kk * 2048, Q_CHUNK, 1024);
          // Each warpgroup packs its 32 query columns into the first 16 TMEM
          // columns of its own 32-column fp32 half, so the other warpgroup's
          // unread scores are never overwritten: K-steps 0-1 read [0,16),
          // K-steps 2-3 read [32,48) of the buffer.
          mma_ts(tmem + d_col, tmem + a_col + (kk >> 1) * 32 + (kk & 1) * 8, bd, ID_DV,
                 (acc || kk > 0) ? 1u : 0u);
        }
      };
      // S^T is double-buffered in TMEM, so S^T(it+2) is issued as soon as
      // dV(it) has read P^T(it) from the same buffer; the conversion
      // warpgroups never wait for the MMA chain of the previous tile.
      auto issue_s = [&](int jt) {
        issue_t(T_S + (jt & 1) * 64, k_base, q_base + (jt % NQS) * KC * Q_CHUNK);
        mma_commit(&s_ready[jt & 1]);
        BWD_TRACE(true, 1, jt);
      };
      bool ok = mbar_wait(kv_full, 0, 0x601) && mbar_wait(&q_full[0], 0, 0x602);
      if (ok) {
        tc_fence_after();
        issue_s(0);
        issue_t(T_DP, v_base, do_base);
        mma_commit(dp_ready);
        if (n > 1) {
          ok = mbar_wait(&q_full[1], 0, 0x609);
          tc_fence_after();
          if (ok) issue_s(1);
        }
      }
      for (int it = 0; ok && it < n; ++it) {
        const int s = it % NQS;
        const uint32_t ph = it & 1;
        if (!mbar_wait(&p_ready[it & 1], (it >> 1) & 1, 0x603)) { ok = false; break; }
        BWD_TRACE(true, 2, it);
        tc_fence_after();
        issue_acc(T_DV, T_S + (it & 1) * 64, do_base + s * KC * Q_CHUNK, it > 0);
        mma_commit(dv_done);
        BWD_TRACE(true, 3, it);
        if (!mbar_wait(ds_ready, ph, 0x606)) { ok = false; break; }
        BWD_TRACE(true, 4, it);
        tc_fence_after();
        if (it + 1 < n) {
          // dS^T(it) lives in S buffer it & 1, so dP^T(it+1) may overwrite
          // dP^T(it) as soon as both warpgroups have read it (ds_ready).
          issue_t(T_DP, v_base, do_base + ((it + 1) % NQS) * KC * Q_CHUNK);
          mma_commit(dp_ready);
        }
        issue_acc(T_DK, T_S + (it & 1) * 64 + 16, q_base + s * KC * Q_CHUNK, it > 0);
        mma_commit(dk_done);
        BWD_TRACE(true, 5, it);
        if (it > 0 && !mbar_wait(dq_free, (it - 1) & 1, 0x607)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t a = smem_desc_sw128(k_base + kk * 2048, KV_CHUNK, 1024);
          const uint64_t bd = smem_desc_sw128(ds_base + (it & 1) * DS_BYTES + kk * 2048, DS_BYTES, 1024);
          mma_ss(tmem + T_DQ, a, bd, ID_DQ, kk > 0);
        }
        mma_commit(dq_ready);
        BWD_TRACE(true, 6, it);
        mma_commit(&q_empty[s]);
        if (it + 2 < n) {
          // S^T(it+2) overwrites P^T(it) and dS^T(it) in buffer it & 1:
          // dV(it) and dK(it) must have read them.
          if (!mbar_wait(&q_full[(it + 2) % NQS], ((it + 2) / NQS) & 1, 0x604) ||
              !mbar_wait(dk_done, ph, 0x605)) { ok = false; break; }
          tc_fence_after();
          issue_s(it + 2);
        }
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------- dQ reducer --
    // Adds each staged 64-row dQ tile into the fp32 dQ buffer (rows are
    // contiguous there) with one bulk reduction. Tiles are staged one tile
    // late, so the staging buffer is normally read by the time it is reused.
    reg_dealloc<72>();
    if (lane == 0) {
      for (int it = 0; it < n; ++it) {
        if (!mbar_wait(red_full, it & 1, 0x901)) break;
        const int m0 = (i0 + it) * BM;
        const int rows = min(BM, p.N - m0);
        bulk_reduce_add_f32(p.dq_acc + ((int64_t)bh * p.N + m0) * D,
                            reinterpret_cast<const float*>(smem + RED_OFF), rows * D * 4);
        bulk_commit();
        bulk_wait_read();  // the staging tile may be rewritten once this has read it
        mbar_arrive(red_free);
      }
      bulk_wait_all();  // every reduction has landed before the CTA exits
    }
  } else if (warp < 4) {
    reg_dealloc<72>();
  } else {
    // ------------------------------------------------------------------------
    // Two warpgroups split the 64 query columns of each tile (32 each):
    // thread = key (TMEM lane) for P^T / dS^T, then thread = head-dim index
    // for its half of the dQ^T columns. Epilogue: warpgroup 1 writes dV,
    // warpgroup 2 writes dK.
    reg_alloc<216>();
    const int half = warp >> 3;                  // 0: q cols [0,32), 1: [32,64)
    const int r = (threadIdx.x & 127);           // TMEM lane: key, then head-dim index
    const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const int key = kv0 + r;
    const float sl2 = p.scale_log2;
    const int cb = half * 32;                    // first query column of this half
    // dQ^T columns [cb, cb+32) of tile jt: thread = head-dim index r. The 32
    // query rows are staged [q][d] in shared memory; warp 2 adds the whole
    // 64-row tile into the fp32 dQ buffer with one bulk reduction.
    auto stage_dq = [&](int jt) -> bool {
      if (!mbar_wait_warp(dq_ready, jt & 1, 0x801)) return false;
      BWD_TRACE(r == 0 && half == 0, 11, jt);
      tc_fence_after();
      uint32_t qv[32];
      tmem_ld32(lane_addr + T_DQ + cb, qv);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(dq_free);
      if (jt >= 1 && !mbar_wait_warp(red_free, (jt - 1) & 1, 0x802)) return false;
      float* stage = reinterpret_cast<float*>(smem + RED_OFF) + half * 32 * D;
#pragma unroll
      for (int c = 0; c < 32; ++c) stage[c * D + r] = __uint_as_float(qv[c]) * p.scale;
      fence_proxy_async_smem();
      mbar_arrive(red_full);
      BWD_TRACE(r == 0 && half == 0, 12, jt);
      return true;
    };
    bool ok = true;
    for (int it = 0; it < n; ++it) {
      const uint32_t ph = it & 1;
      const int m0 = (i0 + it) * BM;
      const float* st = stats + (it % NQS) * 2 * BM;
      const uint32_t sbuf = T_S + (it & 1) * 64;
      if (!mbar_wait_warp(&stat_full[it % NQS], (it / NQS) & 1, 0x705)) { ok = false; break; }
      if (!mbar_wait_warp(&s_ready[it & 1], (it >> 1) & 1, 0x701)) { ok = false; break; }
      BWD_TRACE(r == 0 && half == 0, 7, it);
      tc_fence_after();
      uint32_t sv[32];
      tmem_ld32(lane_addr + sbuf + cb, sv);
      tmem_ld_wait();
      // Masks: causal (q < key), and rows/columns past the sequence end.
      const bool need_mask = (m0 + BM > p.N) || (kv0 + BN > p.N) || (p.causal && m0 < kv0 + BN);
      const int qlo = p.causal ? key : 0;  // first valid q for this key
      float pf[32];
      uint32_t pk[16];
#pragma unroll
      for (int cc = 0; cc < 16; ++cc) {
        const int c0 = cb + 2 * cc;
        const float2 l2 = *reinterpret_cast<const float2*>(st + c0);  // shared broadcast
        float p0 = ex2(fmaf(__uint_as_float(sv[2 * cc]), sl2, -l2.x));
        float p1 = ex2(fmaf(__uint_as_float(sv[2 * cc + 1]), sl2, -l2.y));
        if (need_mask) {
          const int q0 = m0 + c0;
          if (key >= p.N || q0 >= p.N || q0 < qlo) p0 = 0.f;
          if (key >= p.N || q0 + 1 >= p.N || q0 + 1 < qlo) p1 = 0.f;
        }
        pf[2 * cc] = p0;
        pf[2 * cc + 1] = p1;
        pk[cc] = pack2<FMT>(p0, p1);
      }
      tmem_st16(lane_addr + sbuf + half * 32, pk);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_ready[it & 1]);
      BWD_TRACE(r == 0 && half == 0, 8, it);

      if (!mbar_wait_warp(dp_ready, ph, 0x702)) { ok = false; break; }
      BWD_TRACE(r == 0 && half == 0, 9, it);
      tc_fence_after();
      tmem_ld32(lane_addr + T_DP + cb, sv);
      tmem_ld_wait();
      uint32_t dsk[16];
#pragma unroll
      for (int cc = 0; cc < 16; ++cc) {
        const float2 ds2 = *reinterpret_cast<const float2*>(st + BM + cb + 2 * cc);
        dsk[cc] = pack2<FMT>(pf[2 * cc] * (__uint_as_float(sv[2 * cc]) - ds2.x),
                             pf[2 * cc + 1] * (__uint_as_float(sv[2 * cc + 1]) - ds2.y));
      }
      tmem_st16(lane_addr + sbuf + half * 32 + 16, dsk);  // beside P^T, in the S buffer
      // dS^T row half -> shared (128-byte swizzle) for the dQ^T GEMM, once the
      // previous dQ^T GEMM has finished reading the buffer.
      // dS^T buffer it & 1 was last read by dQ^T(it-2), which stage_dq(it-2)
      // waited for during the previous tile.
      {
        uint8_t* rowp = sDS + (it & 1) * DS_BYTES + r * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int chunk = half * 4 + c;
          *reinterpret_cast<uint4*>(rowp + ((chunk ^ (r & 7)) << 4)) =
              make_uint4(dsk[4 * c], dsk[4 * c + 1], dsk[4 * c + 2], dsk[4 * c + 3]);
        }
      }
      fence_proxy_async_smem();
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(ds_ready);
      BWD_TRACE(r == 0 && half == 0, 10, it);
      // The previous tile's dQ^T (complete by now) is staged while dK(it) and
      // dQ^T(it) run on the tensor cores.
      if (it > 0 && !stage_dq(it - 1)) { ok = false; break; }

    }
    if (ok && !stage_dq(n - 1)) ok = false;
    // Epilogue: warpgroup 1 writes this key's dV row, warpgroup 2 its dK row.
    if (ok && mbar_wait_warp(dk_done, (n - 1) & 1, 0x704)) {
      tc_fence_after();
      // tcgen05.ld is warp-collective: every lane loads, only valid keys store.
      const bool store = key < p.N;
      const uint32_t col = half == 0 ? T_DV : T_DK;
      const float mul = half == 0 ? 1.f : p.scale;
      uint8_t* dst = half == 0
          ? reinterpret_cast<uint8_t*>(p.dv) + 2 * (b * p.sdv_b + h * p.sdv_h + (int64_t)key * p.sdv_n)
          : reinterpret_cast<uint8_t*>(p.dk) + 2 * (b * p.sdk_b + h * p.sdk_h + (int64_t)key * p.sdk_n);
#pragma unroll
      for (int i = 0; i < D / 32; ++i) {
        uint32_t v[32];
        tmem_ld32(lane_addr + col + 32 * i, v);
        tmem_ld_wait();
        uint32_t pk2[16];
#pragma unroll
        for (int cc = 0; cc < 16; ++cc)
          pk2[cc] = pack2<FMT>(__uint_as_float(v[2 * cc]) * mul, __uint_as_float(v[2 * cc + 1]) * mul);
        if (store) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + 64 * i);
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4)
            d4[v4] = make_uint4(pk2[4 * v4], pk2[4 * v4 + 1], pk2[4 * v4 + 2], pk2[4 * v4 + 3]);
        }
      }
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
  if (D != fa_bwd::D) return false;
  if (B * H > 65535 || N >= (1LL << 30)) return false;
  if (!tma_ok(q, B, H, N, sq, 2) || !tma_ok(k, B, H, N, sk, 2) || !tma_ok(v, B, H, N, sv, 2) ||
      !tma_ok(dout, B, H, N, sdo, 2))
    return false;
  // dK/dV rows are written with 16-byte stores.
  for (auto pr : {std::make_pair(dk, sdk), std::make_pair(dv, sdv)}) {
    const int64_t* s = pr.second;
    if (!aligned16(pr.first) || s[3] != 1 || (s[2] * 2) % 16 || (s[1] * 2) % 16 || (s[0] * 2) % 16)
      return false;
  }
  return true;
}

template <int FMT>
static int launch_fa_bwd(const void* q, const void* k, const void* v, const void* dout,
                         const float* lse, void* dk, void* dv, int64_t B, int64_t H, int64_t N,
                         const int64_t* sq, const int64_t* sk, const int64_t* sv,
                         const int64_t* sdo, const int64_t* sdk, const int64_t* sdv, float scale,
                         int causal, int dtype, const float* dsum, float* dq_acc,
                         cudaStream_t st) {
  using namespace fa_bwd;
  CUtensorMap mq, mk, mv, mdo;
  int rc = make_bhnd_map(&mq, q, dtype, B, H, N, D, sq, 64, BM);
  if (!rc) rc = make_bhnd_map(&mdo, dout, dtype, B, H, N, D, sdo, 64, BM);
  if (!rc) rc = make_bhnd_map(&mk, k, dtype, B, H, N, D, sk, 64, BN);
  if (!rc) rc = make_bhnd_map(&mv, v, dtype, B, H, N, D, sv, 64, BN);
  if (rc) return rc;
  Params p;
  p.lse = lse; p.dsum = dsum; p.dq_acc = dq_acc; p.dk = dk; p.dv = dv;
  p.sdk_b = sdk[0]; p.sdk_h = sdk[1]; p.sdk_n = sdk[2];
  p.sdv_b = sdv[0]; p.sdv_h = sdv[1]; p.sdv_n = sdv[2];
  p.H = (int)H; p.N = (int)N;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  auto kern = fa_bwd_kernel<FMT>;
  LSB_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM),
              "attn_bwd_tc smem attribute");
  dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)(B * H));
  kern<<<grid, THREADS, SMEM, st>>>(mq, mk, mv, mdo, p);
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
  int rc = bf ? launch_dsum<__nv_bfloat16>(o, dout, dsum, B, H, N, D, S4(so), S4(sdo), st)
              : launch_dsum<__half>(o, dout, dsum, B, H, N, D, S4(so), S4(sdo), st);
  if (rc) return rc;
  LSB_CUDA_OK(cudaMemsetAsync(dq_acc, 0, sizeof(float) * (size_t)(B * H * N * D), st),
              "attn_bwd dQ accumulator memset");
  rc = bf ? launch_fa_bwd<1>(q, k, v, dout, lse, dk, dv, B, H, N, sq, sk, sv, sdo, sdk, sdv, scale,
                             causal, dtype, dsum, dq_acc, st)
          : launch_fa_bwd<0>(q, k, v, dout, lse, dk, dv, B, H, N, sq, sk, sv, sdo, sdk, sdv, scale,
                             causal, dtype, dsum, dq_acc, st);
  if (rc) return rc;
  return bf ? launch_dq_cast<__nv_bfloat16>(dq_acc, dq, B, H, N, D, S4(sdq), st)
            : launch_dq_cast<__half>(dq_acc, dq, B, H, N, D, S4(sdq), st);
}

#ifdef LSB_BWD_TRACE
extern "C" LSB_API int lsb_bwd_trace_read(long long* out) {
  return (int)cudaMemcpyFromSymbol(out, fa_bwd::g_bwd_trace, sizeof(fa_bwd::g_bwd_trace));
}
#endif

int attn_bwd_tc_device_error() {
  int e = 0;
  cudaMemcpyFromSymbol(&e, sm100::g_lsb_device_error, sizeof(int));
  return e;
}

}  // namespace lsb
