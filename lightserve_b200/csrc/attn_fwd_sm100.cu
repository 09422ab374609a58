// FlashAttention forward on the 5th-generation tensor cores (sm_100a).
//
// Same arithmetic as lightserve's _flash_attn_fwd_kernel /
// _flash_attn_fwd_lse_kernel (kernels/flash_attention.py:84-179,
// kernels/flash_attention_backward.py:88-169): S = Q K^T * scale with the
// causal and sequence-end masks, online softmax with fp32 row statistics,
// P rounded to the input dtype before P V, O = acc / l, L = m + ln(l).
//
// B200 design (one CTA per 256 query rows of one (batch, head)):
//  * warp 0: TMA producer. Q tiles once, then K and V tiles of 128 keys into a
//    2-stage ring (128-byte-swizzled boxes of 64 head-dim columns).
//  * warp 1: TMEM owner and single-thread MMA issuer. Two query tiles of 128
//    rows share each K/V tile: S_t = Q_t K^T (SS MMA, fp32 in TMEM) and
//    O_t += P_t V (TS MMA: P read from TMEM, V from shared memory).
//  * warpgroups 1 and 2: softmax for query tile 0 and 1, one thread per row
//    (TMEM lane). Each thread loads its 128 scores with tcgen05.ld, takes the
//    row max, exponentiates with ex2 on log2(e)-prescaled scores, writes P as
//    packed 16-bit pairs over the first 64 columns of its S buffer, and
//    rescales O in TMEM only when the running max grew by more than 2^8
//    (otherwise the stale max is kept; values stay within fp32/bf16 range).
//  * TMEM: S0 [0,128), S1 [128,256), O0 [256,384), O1 [384,512) columns.
//  * MMA order per K/V tile j: PV_0(j), QK_0(j+1), PV_1(j), QK_1(j+1), so each
//    softmax warpgroup's work overlaps the other tile's two GEMMs.
//  * Causal: query tile t of CTA c stops at its diagonal K/V tile; CTAs are
//    issued heaviest first.
//  * Every mbarrier wait is bounded (sm100.cuh); on a timeout the kernel
//    records an error code, skips the rest of its work, frees TMEM and exits.
#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace lsb {

namespace fa_fwd {

constexpr int BM = 128;      // query rows per tile (= TMEM lanes)
constexpr int BN = 128;      // keys per K/V tile
constexpr int TILES = 2;     // query tiles per CTA
constexpr int NS = 2;        // K/V ring stages
constexpr int THREADS = 384;
constexpr int CHUNK_BYTES = 128 * 128;  // one [128 rows][64 cols] 16-bit box
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units

template <int D>
struct Smem {
  static constexpr int KC = D / 64;  // 64-column chunks per row
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + TILES * KC * CHUNK_BYTES;
  static constexpr int V_OFF = K_OFF + NS * KC * CHUNK_BYTES;
  static constexpr int BAR_OFF = V_OFF + NS * KC * CHUNK_BYTES;
  // barriers: q_full, k_full[NS], v_full[NS], kv_empty[NS], s_full[2], p_full[2], pv_done[2]
  static constexpr int NBAR = 1 + 3 * NS + 3 * TILES;
  static constexpr int TMEM_SLOT_OFF = BAR_OFF + NBAR * 8;
  static constexpr int BYTES = TMEM_SLOT_OFF + 16;
  static constexpr int ALLOC = BYTES + 1024;  // slack for 1024-byte alignment
};

struct Params {
  void* o;
  float* lse;
  int64_t so_b, so_h, so_n;
  int H, N;
  int num_q_ctas;
  float scale_log2;
  int causal;
};

using namespace sm100;

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
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

template <int D, int FMT>
__global__ void __launch_bounds__(THREADS, 1)
fa_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
              const __grid_constant__ CUtensorMap tv, const Params p) {
  using L = Smem<D>;
  constexpr int KC = L::KC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = bars + 1 + NS;
  uint64_t* kv_empty = bars + 1 + 2 * NS;
  uint64_t* s_full = bars + 1 + 3 * NS;
  uint64_t* p_full = s_full + TILES;
  uint64_t* pv_done = p_full + TILES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::TMEM_SLOT_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int c = p.causal ? (p.num_q_ctas - 1 - (int)blockIdx.x) : (int)blockIdx.x;
  const int q0 = c * (TILES * BM);
  const int nkv_all = (p.N + BN - 1) / BN;
  int nkv_t[TILES];
#pragma unroll
  for (int t = 0; t < TILES; ++t) {
    const int qt0 = q0 + t * BM;
    nkv_t[t] = qt0 >= p.N ? 0 : (p.causal ? min(nkv_all, qt0 / BN + 1) : nkv_all);
  }
  const int nkv = max(nkv_t[0], nkv_t[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < TILES; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], BM);
      mbar_init(&pv_done[t], 1);
    }
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

  uint8_t* sQ = smem + L::Q_OFF;
  uint8_t* sK = smem + L::K_OFF;
  uint8_t* sV = smem + L::V_OFF;

  // Register split: 384 threads x 168 at launch = 128 x 56 (TMA/MMA warpgroup)
  // + 256 x 224 (softmax warpgroups).
  // (setmaxnreg sits at the top of each role's branch so ptxas budgets each.)
  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    reg_dealloc<56>();
    if (lane == 0) {
      prefetch_tmap(&tq); prefetch_tmap(&tk); prefetch_tmap(&tv);
      mbar_arrive_expect_tx(q_full, TILES * KC * CHUNK_BYTES);
      for (int t = 0; t < TILES; ++t)
        for (int kc = 0; kc < KC; ++kc)
          tma_load_4d(sQ + (t * KC + kc) * CHUNK_BYTES, &tq, q_full, kc * 64, q0 + t * BM, h, b);
      for (int j = 0; j < nkv; ++j) {
        const int s = j % NS;
        if (j >= NS && !mbar_wait(&kv_empty[s], ((j / NS) - 1) & 1, 0x101)) break;
        mbar_arrive_expect_tx(&k_full[s], KC * CHUNK_BYTES);
        for (int kc = 0; kc < KC; ++kc)
          tma_load_4d(sK + (s * KC + kc) * CHUNK_BYTES, &tk, &k_full[s], kc * 64, j * BN, h, b);
        mbar_arrive_expect_tx(&v_full[s], KC * CHUNK_BYTES);
        for (int kc = 0; kc < KC; ++kc)
          tma_load_4d(sV + (s * KC + kc) * CHUNK_BYTES, &tv, &v_full[s], kc * 64, j * BN, h, b);
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issue --
    reg_dealloc<56>();
    if (lane == 0) {
      constexpr uint32_t IDESC_QK = idesc_f16(BM, BN, FMT, 0, 0);
      constexpr uint32_t IDESC_PV = idesc_f16(BM, D, FMT, 0, 1);
      const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK), v_base = smem_u32(sV);
      auto issue_qk = [&](int t, int j) {
        const int s = j % NS;
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
      auto issue_pv = [&](int t, int j) {
        const int s = j % NS;
        const uint32_t d_tmem = tmem + 256 + t * 128;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t bd =
              smem_desc_sw128(v_base + (s * KC) * CHUNK_BYTES + kk * 2048, CHUNK_BYTES, 1024);
          mma_ts(d_tmem, tmem + t * 128 + kk * 8, bd, IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&pv_done[t]);
      };
      bool ok = mbar_wait(q_full, 0, 0x201) && (nkv == 0 || mbar_wait(&k_full[0], 0, 0x202));
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < TILES; ++t)
          if (nkv_t[t] > 0) issue_qk(t, 0);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const int s = j % NS;
        if (!mbar_wait(&v_full[s], (j / NS) & 1, 0x203)) { ok = false; break; }
        for (int t = 0; t < TILES; ++t) {
          if (j >= nkv_t[t]) continue;
          if (!mbar_wait(&p_full[t], j & 1, 0x204)) { ok = false; break; }
          tc_fence_after();
          issue_pv(t, j);
          if (j + 1 < nkv_t[t]) {
            const int s1 = (j + 1) % NS;
            // S_t is overwritten by the next QK: wait until PV_t(j) has read P_t.
            if (!mbar_wait(&k_full[s1], ((j + 1) / NS) & 1, 0x205) ||
                !mbar_wait(&pv_done[t], j & 1, 0x206)) { ok = false; break; }
            tc_fence_after();
            issue_qk(t, j + 1);
          }
        }
        mma_commit(&kv_empty[s]);
      }
    }
  } else if (warp < 4) {
    reg_dealloc<56>();  // warps 2-3: idle members of the TMA/MMA warpgroup
  } else {
    // ------------------------------------------------------------- softmax --
    reg_alloc<224>();
    const int t = (warp >> 2) - 1;
    const int row = threadIdx.x - 128 * (t + 1);          // TMEM lane of this thread
    const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const int qt0 = q0 + t * BM;
    const int row_g = qt0 + row;
    const float sl2 = p.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv_t[t]; ++j) {
      if (!mbar_wait_warp(&s_full[t], j & 1, 0x301)) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[4][32];
#pragma unroll
      for (int i = 0; i < 4; ++i) tmem_ld32(lane_addr + t * 128 + 32 * i, sr[i]);
      tmem_ld_wait();
      const int kv0 = j * BN;
      // Only the diagonal tile (causal) and the tile holding position N-1 need masks.
      const bool need_mask = (kv0 + BN > p.N) || (p.causal && kv0 + BN - 1 > qt0);
      const int lim = min(p.N, p.causal ? row_g + 1 : p.N) - kv0;  // valid columns < lim
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
      // row-sum steps; the exponentials go to MUFU.EX2.
      float2 l2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                      make_float2(0.f, 0.f)};
      const float2 sl2_2 = make_float2(sl2, sl2), negm2 = make_float2(-m_use, -m_use);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
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
        for (int cc = 0; cc < 16; ++cc) sr[i >> 1][(i & 1) * 16 + cc] = pk[cc];
      }
      {
        const float2 a2 = __fadd2_rn(__fadd2_rn(l2[0], l2[1]), __fadd2_rn(l2[2], l2[3]));
        l += a2.x + a2.y;
      }
      tmem_st32(lane_addr + t * 128, sr[0]);
      tmem_st32(lane_addr + t * 128 + 32, sr[1]);
      // tcgen05.ld/st are warp-collective: if any row of the warp rescales,
      // the whole warp runs the loop (alpha is 1 for rows that do not).
      if (__any_sync(0xffffffffu, rescale && j > 0)) {
        if (!(rescale && j > 0)) alpha = 1.f;
#pragma unroll
        for (int i = 0; i < D / 32; ++i) {
          uint32_t ov[32];
          tmem_ld32(lane_addr + 256 + t * 128 + 32 * i, ov);
          tmem_ld_wait();
#pragma unroll
          for (int cc = 0; cc < 32; ++cc) ov[cc] = __float_as_uint(__uint_as_float(ov[cc]) * alpha);
          tmem_st32(lane_addr + 256 + t * 128 + 32 * i, ov);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }
    if (ok && nkv_t[t] > 0 && mbar_wait_warp(&pv_done[t], (nkv_t[t] - 1) & 1, 0x302)) {
      tc_fence_after();
      const float inv_l = 1.0f / l;
      uint8_t* orow = reinterpret_cast<uint8_t*>(p.o) +
                      2 * (b * p.so_b + h * p.so_h + (int64_t)row_g * p.so_n);
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
        if (row_g < p.N) {
          uint4* dst = reinterpret_cast<uint4*>(orow + 64 * i);
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4)
            dst[v4] = make_uint4(pk[4 * v4], pk[4 * v4 + 1], pk[4 * v4 + 2], pk[4 * v4 + 3]);
        }
      }
      if (p.lse != nullptr && row_g < p.N)
        p.lse[(int64_t)bh * p.N + row_g] = (m + __log2f(l)) * 0.6931471805599453f;
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
  if (B * H > 65535 || N >= (1LL << 30)) return false;
  if (!tma_ok(q, B, H, N, sq, 2) || !tma_ok(k, B, H, N, sk, 2) || !tma_ok(v, B, H, N, sv, 2))
    return false;
  // Output rows are written with 16-byte stores.
  if (!aligned16(o) || so[3] != 1 || (so[2] * 2) % 16 || (so[1] * 2) % 16 || (so[0] * 2) % 16)
    return false;
  return true;
}

template <int D, int FMT>
static int launch_fa_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                         int64_t B, int64_t H, int64_t N, const int64_t* sq, const int64_t* sk,
                         const int64_t* sv, const int64_t* so, float scale, int causal,
                         int dtype, cudaStream_t st) {
  using namespace fa_fwd;
  CUtensorMap mq, mk, mv;
  int rc = make_bhnd_map(&mq, q, dtype, B, H, N, D, sq, 64, BM);
  if (!rc) rc = make_bhnd_map(&mk, k, dtype, B, H, N, D, sk, 64, BN);
  if (!rc) rc = make_bhnd_map(&mv, v, dtype, B, H, N, D, sv, 64, BN);
  if (rc) return rc;
  Params p;
  p.o = o; p.lse = lse;
  p.so_b = so[0]; p.so_h = so[1]; p.so_n = so[2];
  p.H = (int)H; p.N = (int)N;
  p.num_q_ctas = (int)((N + TILES * BM - 1) / (TILES * BM));
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  const int smem = Smem<D>::ALLOC;
  auto kern = fa_fwd_kernel<D, FMT>;
  LSB_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
              "attn_fwd_tc smem attribute");
  dim3 grid((unsigned)p.num_q_ctas, (unsigned)(B * H));
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

int attn_fwd_tc_device_error() {
  int e = 0;
  cudaMemcpyFromSymbol(&e, sm100::g_lsb_device_error, sizeof(int));
  return e;
}

}  // namespace lsb
