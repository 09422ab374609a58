// Weight-streaming linear layer for decode batches on the 5th-generation
// tensor cores (sm_100a): Y[S, N] = X[S, K] @ W[K, N], with W supplied
// transposed (W^T [N, K], K contiguous) and S <= 128 tokens.
//
// The weight is packed once (lsb_linear_pack) into tiles of 128 features x
// 64 of K, each 16 KiB contiguous and already in the 128-byte-swizzled
// K-major layout the MMA reads, so every weight load is one sequential 16 KiB
// bulk copy (a strided 2-D tile would touch 128 DRAM rows 4-11 KiB apart).
//
// Replaces the `x @ w` projections of lightserve's decode step
// (model/minimal_llama.py:216-234 q/k/v/o and the SwiGLU FFN, :249 lm_head),
// which lightserve computes with torch.matmul or its Triton tiled_matmul
// (kernels/tiled_matmul.py:55-151): fp32 accumulation of bf16/fp16 products,
// one rounding to the output dtype.
//
// At decode batch sizes the whole cost is streaming W from HBM once (953 MB
// per step at config 5); the arithmetic is tiny. So:
//  * Weight tiles are the MMA's A operand (M = 128 output features per tile),
//    X is the B operand (N = S padded to a multiple of 32, at most 128),
//    D^T = W^T X^T accumulates in TMEM (128 lanes x S columns, fp32).
//  * Split-K inside a thread-block cluster: the s CTAs of a cluster share
//    each 128-feature tile, CTA r streaming the r-th of s equal slices of K.
//    Their fp32 partials meet in distributed shared memory: thread = feature
//    row sends its row straight from registers to the cluster CTA that owns
//    the row (rows [128 q / s, 128 (q + 1) / s) belong to CTA q) with
//    st.async, which completes on that CTA's mbarrier; CTA q adds the s
//    slices it received in rank order (the result does not depend on timing)
//    and writes its rows of Y. With s = 1 the epilogue writes Y from
//    registers. Clusters are persistent over tiles (tile = cluster id +
//    k * clusters). s and the cluster count are chosen on the host so that
//    every SM streams about the same number of weight bytes (for example
//    8 x 16 tiles for the 2048 x 2048 o projection, 3 x 48 for the fused
//    q/k/v); the shared memory not needed to receive partials deepens the
//    weight ring.
//  * warp 0 issues TMA loads through a ring of stages (weights 16 KiB + X per
//    stage), warp 1 owns TMEM and issues tcgen05.mma, warps 4-7 run the
//    epilogue (thread = TMEM lane = output feature) from one of two TMEM
//    accumulators while the next tile accumulates in the other.
//  * Programmatic dependent launch: the weight loads of the first stages are
//    issued before griddepcontrol.wait, so when the previous kernel of the
//    stream lets dependents start early the weight stream overlaps its tail;
//    X (produced by that kernel) is loaded only after the wait.
//  * Every mbarrier wait is bounded (sm100.cuh): a wait that gives up records
//    an error code, the kernel skips the rest of its work, frees TMEM and
//    returns. No TMA load here uses cluster multicast.
#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace lsb {
namespace lin {

using namespace sm100;

constexpr int BM = 128;            // output features per tile (TMEM lanes)
constexpr int BK = 64;             // K per stage (one 128-byte swizzle row)
constexpr int W_BYTES = BM * BK * 2;
constexpr int THREADS = 256;
constexpr int MAX_STAGES = 12;
constexpr int SMEM_BUDGET = 220 * 1024;
constexpr int MAX_SPLIT = 8;

// Rows [row_lo(r), row_lo(r + 1)) of a tile are reduced by cluster rank r
// (multiples of 4).
__host__ __device__ constexpr int row_lo(int r, int split) { return (r * (BM / 4) / split) * 4; }

// Shared memory: the TMA ring (stages of W + X), then the receive buffer
// (split > 1 only), then barriers. Sizes depend on SP and the split, so the
// host computes them (linear_layout) and passes them in Params.
struct Params {
  const uint8_t* w_packed;
  void* y;
  int64_t ldy;
  int S, N, n_tiles, kc, split, clusters;
  int stages, stage_bytes, recv_off, bar_off;
};


__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ void arrive_remote(uint32_t cluster_bar_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar_addr)
               : "memory");
}

__device__ __forceinline__ bool try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait (acquire at cluster scope) on a barrier peers arrive on.
__device__ __forceinline__ bool wait_cluster(uint64_t* bar, uint32_t parity, int code) {
  if (try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (!try_wait_cluster(bar, parity)) {
    if (clock64() - t0 > LSB_WAIT_CYCLES) {
      atomicCAS(&g_lsb_device_error, 0, code);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}

// OR of `pred` over the 128 epilogue threads (warps 4-7), as a barrier.
__device__ __forceinline__ bool epi_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 q, %1, 0;\n\t"
      "bar.red.or.pred p, 1, 128, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void st_async_v4(uint32_t dst_cluster, uint4 v, uint32_t bar_cluster) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
          dst_cluster),
      "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(bar_cluster)
      : "memory");
}

template <int FMT, int SP>
__global__ void __launch_bounds__(THREADS, 1)
linear_wstream_kernel(const __grid_constant__ CUtensorMap tx, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int NS = p.stages;
  const int STAGE = p.stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* full = bars;
  uint64_t* empty = full + NS;
  uint64_t* acc_full = empty + NS;     // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint64_t* recv_full = acc_empty + 2;  // every slice of this CTA's rows has arrived
  uint64_t* send_ok = recv_full + 1;    // every peer's receive buffer is free again
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(send_ok + 1);
  float* recv = reinterpret_cast<float*>(smem + p.recv_off);  // [split][rows of this rank][SP]

  allow_dependents();  // the next kernel may launch; it waits for this one's completion
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = p.split;
  const int rank = (int)cluster_rank();
  const int cid = blockIdx.x / split;
  // This CTA's slice of every tile's K chunks.
  const int k_lo = (rank * p.kc) / split, k_hi = ((rank + 1) * p.kc) / split;
  const int nk = k_hi - k_lo;
  const int n_my_tiles = cid < p.n_tiles ? (p.n_tiles - 1 - cid) / p.clusters + 1 : 0;
  constexpr uint32_t tmem_cols = SP <= 64 ? 128 : 256;  // two accumulators of SP columns

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], BM);
    }
    mbar_init(recv_full, 1);     // the receiver's expect_tx arrival (+ the bytes)
    mbar_init(send_ok, split);   // one arrival from every receiver
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  if (split > 1) cluster_sync_all();  // peers' barriers are initialised before anyone uses them
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    const int total = n_my_tiles * nk;  // K chunks this CTA streams
    if (lane == 0 && total > 0) {
      prefetch_tmap(&tx);
      auto load_w = [&](int i) {
        const int t = cid + (i / nk) * p.clusters, k = k_lo + i % nk, s = i % NS;
        mbar_arrive_expect_tx(&full[s], STAGE);
        bulk_load(smem + s * STAGE, p.w_packed + ((int64_t)t * p.kc + k) * W_BYTES, W_BYTES, &full[s]);
      };
      auto load_x = [&](int i) {
        const int k = k_lo + i % nk, s = i % NS;
        tma_load_4d(smem + s * STAGE + W_BYTES, &tx, &full[s], k * BK, 0, 0, 0);
      };
      const int pre = min(NS, total);
      for (int i = 0; i < pre; ++i) load_w(i);  // weights do not depend on the previous kernel
      griddep_wait();
      for (int i = 0; i < pre; ++i) load_x(i);
      for (int i = pre; i < total; ++i) {
        if (!mbar_wait(&empty[i % NS], ((i / NS) - 1) & 1, 0x701)) break;
        load_w(i);
        load_x(i);
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issue --
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(BM, SP, FMT, 0, 0);
      const uint32_t base = smem_u32(smem);
      bool ok = true;
      int i = 0;
      for (int j = 0; ok && j < n_my_tiles; ++j) {
        const int b = j & 1;
        // The epilogue has read this accumulator's previous tile out.
        if (j >= 2 && !mbar_wait(&acc_empty[b], ((j >> 1) - 1) & 1, 0x702)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + b * SP;
        for (int kk4 = 0; kk4 < nk; ++kk4, ++i) {
          const int s = i % NS;
          if (!mbar_wait(&full[s], (i / NS) & 1, 0x703)) { ok = false; break; }
          tc_fence_after();
          const uint32_t wa = base + s * STAGE, xa = wa + W_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_ss(d_tmem, smem_desc_sw128(wa + kk * 32, 16, 1024),
                   smem_desc_sw128(xa + kk * 32, 16, 1024), idesc, (kk4 == 0 && kk == 0) ? 0u : 1u);
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[b]);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue --
    griddep_wait();  // Y may alias memory the previous kernel still reads
    const int et = threadIdx.x - 128;  // TMEM lane = feature row within the tile
    const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const int r0 = row_lo(rank, split), r1 = row_lo(rank + 1, split);
    const int nr = r1 - r0;  // rows of every tile this CTA reduces
    // The rank that reduces this thread's row, and where the row goes there.
    int owner = 0;
    while (owner + 1 < split && et >= row_lo(owner + 1, split)) ++owner;
    const int o0 = row_lo(owner, split), onr = row_lo(owner + 1, split) - o0;
    const uint32_t dst_row = (uint32_t)(((rank * onr) + (et - o0)) * SP * 4);
    const uint32_t owner_recv = map_rank(smem_u32(recv), (uint32_t)owner);
    const uint32_t owner_bar = map_rank(smem_u32(recv_full), (uint32_t)owner);
    uint16_t* yb = reinterpret_cast<uint16_t*>(p.y);
    for (int j = 0; j < n_my_tiles; ++j) {
      const int b = j & 1;
      const int t = cid + j * p.clusters;
      // The four epilogue warps leave together if any of their bounded waits
      // gave up (they meet at named barriers below).
      if (epi_any(!mbar_wait_warp(&acc_full[b], (j >> 1) & 1, 0x704))) break;
      tc_fence_after();
      uint32_t acc[SP];
#pragma unroll
      for (int c = 0; c < SP; c += 32) {
        uint32_t r[32];
        tmem_ld32(lane_addr + b * SP + c, r);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 32; ++q) acc[c + q] = r[q];
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
      if (split == 1) {
        // Whole K in this CTA: row `et` of the tile straight to Y.
        const int n = t * BM + et;
        if (n < p.N) {
#pragma unroll
          for (int tok = 0; tok < SP; ++tok) {
            if (tok < p.S) {
              const float f = __uint_as_float(acc[tok]);
              const uint32_t h = FMT == 1 ? pack_bf16(f, 0.f) : pack_f16(f, 0.f);
              yb[(int64_t)tok * p.ldy + n] = (uint16_t)h;
            }
          }
        }
        continue;
      }
      // Every peer's receive buffer is free (they reduced the previous tile).
      bool ok = true;
      if (et == 0 && j > 0) ok = wait_cluster(send_ok, (j - 1) & 1, 0x705);
      if (epi_any(!ok)) break;
      // This tile's slices of this CTA's rows: `split` senders x nr rows.
      if (et == 0) mbar_arrive_expect_tx(recv_full, (uint32_t)(split * nr * SP * 4));
#pragma unroll
      for (int c = 0; c < SP / 4; ++c)
        st_async_v4(owner_recv + dst_row + 16 * c,
                    make_uint4(acc[4 * c], acc[4 * c + 1], acc[4 * c + 2], acc[4 * c + 3]), owner_bar);
      if (epi_any(!mbar_wait_warp(recv_full, j & 1, 0x706))) break;
      // Rows [r0, r1) of the tile: the split slices summed in rank order.
      const int ng = SP / 4;  // 4-token groups per row
      for (int e = et; e < nr * ng; e += 128) {
        const int rl = e / ng, tg = e - rl * ng;
        float4 sum = *reinterpret_cast<const float4*>(recv + rl * SP + 4 * tg);
        for (int c = 1; c < split; ++c) {
          const float4 v = *reinterpret_cast<const float4*>(recv + (c * nr + rl) * SP + 4 * tg);
          sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
        }
        const int n = t * BM + r0 + rl;
        if (n < p.N) {
          const float sv[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int tok = 4 * tg + u;
            if (tok < p.S) {
              const uint32_t h = FMT == 1 ? pack_bf16(sv[u], 0.f) : pack_f16(sv[u], 0.f);
              yb[(int64_t)tok * p.ldy + n] = (uint16_t)h;
            }
          }
        }
      }
      // Tell every sender that the receive buffer is free, if a later tile
      // uses it (a peer may already have exited otherwise).
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (j + 1 < n_my_tiles && et < split)
        arrive_remote(map_rank(smem_u32(send_ok), (uint32_t)et));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
  // Every st.async into this CTA's receive buffer has completed (its last
  // tile waited for them), so it may exit.
}

}  // namespace lin
}  // namespace lsb

using namespace lsb;

namespace {

int64_t linear_s_pad(int64_t S) { return (S + 31) / 32 * 32; }

using LinKern = void (*)(CUtensorMap, lin::Params);

template <int FMT>
LinKern pick_kernel(int sp) {
  switch (sp) {
    case 32: return lin::linear_wstream_kernel<FMT, 32>;
    case 64: return lin::linear_wstream_kernel<FMT, 64>;
    case 96: return lin::linear_wstream_kernel<FMT, 96>;
    default: return lin::linear_wstream_kernel<FMT, 128>;
  }
}

// Shared-memory layout for a padded token count and split; returns the bytes
// to request (with slack for the 1024-byte alignment of the ring).
int linear_layout(int sp, int split, lin::Params* p) {
  p->stage_bytes = lin::W_BYTES + sp * lin::BK * 2;
  const int recv = split > 1 ? (lin::BM + 4 * lin::MAX_SPLIT) * sp * 4 : 0;
  p->stages = std::min(lin::MAX_STAGES, (lin::SMEM_BUDGET - recv) / p->stage_bytes);
  p->recv_off = p->stages * p->stage_bytes;
  p->bar_off = p->recv_off + recv;
  return p->bar_off + (2 * p->stages + 6) * 8 + 16 + 1024;
}

// Clusters of `split` CTAs that fit on the device at once (cached per
// device, kernel and split).
int max_clusters(LinKern kern, int smem, int split, int* out) {
  const int dev = current_device("linear");
  if (dev < 0) return LSB_ERR_CUDA;
  static std::mutex mu;
  static std::atomic<int> cache[kMaxDevices][8][lin::MAX_SPLIT + 1] = {};
  const int ki = [&] {
    const LinKern ks[8] = {lin::linear_wstream_kernel<0, 32>, lin::linear_wstream_kernel<0, 64>,
                           lin::linear_wstream_kernel<0, 96>, lin::linear_wstream_kernel<0, 128>,
                           lin::linear_wstream_kernel<1, 32>, lin::linear_wstream_kernel<1, 64>,
                           lin::linear_wstream_kernel<1, 96>, lin::linear_wstream_kernel<1, 128>};
    for (int i = 0; i < 8; ++i)
      if (ks[i] == kern) return i;
    return 0;
  }();
  int v = cache[dev][ki][split].load(std::memory_order_acquire);
  if (v == 0) {
    std::lock_guard<std::mutex> lock(mu);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)split);
    cfg.blockDim = dim3(lin::THREADS);
    cfg.dynamicSmemBytes = (size_t)smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)split;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    LSB_CUDA_OK(cudaOccupancyMaxActiveClusters(&n, kern, &cfg), "linear cluster occupancy");
    v = n > 0 ? n : -1;
    cache[dev][ki][split].store(v, std::memory_order_release);
  }
  *out = v;
  return LSB_OK;
}

}  // namespace

// Packs W^T [N, K] (row stride ldw) into 16 KiB tiles: tile (t, k) holds
// features [128 t, 128 t + 128) x K columns [64 k, 64 k + 64), row r at byte
// 128 r, its 16-byte chunk c at position c ^ (r % 8) (the 128-byte swizzle),
// zeros past N and K.
template <typename T>
__global__ void linear_pack_kernel(const T* __restrict__ w_t, int64_t ldw, int N, int K, int kc,
                                   int64_t total_chunks, T* __restrict__ packed) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total_chunks;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int pch = (int)(i & 7);          // position of the 16-byte chunk in the row
    const int r = (int)((i >> 3) & 127);   // row within the tile
    const int64_t tile = i >> 10;          // t * kc + k
    const int t = (int)(tile / kc), k = (int)(tile - (int64_t)t * kc);
    const int n = t * lin::BM + r;
    const int c = pch ^ (r & 7);           // logical chunk stored here
    const int k0 = k * lin::BK + c * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (n < N && k0 < K) v = *reinterpret_cast<const uint4*>(w_t + (int64_t)n * ldw + k0);
    reinterpret_cast<uint4*>(packed)[i] = v;
  }
}

extern "C" int64_t lsb_linear_packed_bytes(int64_t N, int64_t K) {
  if (N <= 0 || K <= 0) return 0;
  return ((N + lin::BM - 1) / lin::BM) * ((K + lin::BK - 1) / lin::BK) * (int64_t)lin::W_BYTES;
}

extern "C" int lsb_linear_pack(const void* w_t, int64_t ldw, int64_t N, int64_t K, int dtype,
                               void* packed, int64_t packed_bytes, void* stream) {
  LSB_CHECK_ARG(N >= 0 && K >= 0, "linear_pack: negative size");
  if (N == 0 || K == 0) return LSB_OK;
  LSB_CHECK_ARG(dtype == LSB_DTYPE_BF16 || dtype == LSB_DTYPE_F16, "linear_pack: bf16 or fp16 only");
  LSB_CHECK_ARG(w_t && packed, "linear_pack: null pointer");
  LSB_CHECK_ARG(K % 8 == 0 && ldw % 8 == 0 && ldw >= K && aligned16(w_t) && aligned16(packed),
                "linear_pack: K and ldw must be multiples of 8, 16-byte aligned pointers");
  LSB_CHECK_ARG(N <= 0x7fffffffLL && K <= 0x7fffffffLL, "linear_pack: shape too large");
  const int64_t need = lsb_linear_packed_bytes(N, K);
  LSB_CHECK_ARG(packed_bytes >= need, "linear_pack: %lld bytes needed, got %lld", (long long)need,
                (long long)packed_bytes);
  const int kc = (int)((K + lin::BK - 1) / lin::BK);
  const int64_t chunks = need / 16;
  const unsigned grid = (unsigned)std::min<int64_t>((chunks + 255) / 256, 148 * 16);
  if (dtype == LSB_DTYPE_BF16)
    linear_pack_kernel<__nv_bfloat16><<<grid, 256, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16*)w_t, ldw, (int)N, (int)K, kc, chunks, (__nv_bfloat16*)packed);
  else
    linear_pack_kernel<__half><<<grid, 256, 0, (cudaStream_t)stream>>>(
        (const __half*)w_t, ldw, (int)N, (int)K, kc, chunks, (__half*)packed);
  LSB_CHECK_LAUNCH("linear_pack");
  return LSB_OK;
}

extern "C" int lsb_linear(const void* x, int64_t ldx, const void* w_packed, void* y, int64_t ldy,
                          int64_t S, int64_t N, int64_t K, int dtype, int pdl, void* stream) {
  LSB_CHECK_ARG(S >= 0 && N >= 0 && K >= 0, "linear: negative size");
  if (S == 0 || N == 0) return LSB_OK;
  LSB_CHECK_ARG(S <= 128, "linear: S=%lld tokens above the 128 this kernel serves", (long long)S);
  LSB_CHECK_ARG(K > 0 && K % 8 == 0, "linear: K=%lld must be a positive multiple of 8", (long long)K);
  LSB_CHECK_ARG(dtype == LSB_DTYPE_BF16 || dtype == LSB_DTYPE_F16, "linear: bf16 or fp16 only");
  LSB_CHECK_ARG(x && w_packed && y, "linear: null pointer");
  LSB_CHECK_ARG(aligned16(x) && aligned16(w_packed) && ldx % 8 == 0 && ldx >= K && ldy >= N,
                "linear: x and w_packed need 16-byte aligned bases, x a row stride that is a "
                "multiple of 8 elements and at least K; ldy >= N");
  LSB_CHECK_ARG(N <= 0x7fffffffLL && K <= 0x7fffffffLL, "linear: shape too large");
  lin::Params p;
  p.y = y;
  p.ldy = ldy;
  p.S = (int)S;
  p.N = (int)N;
  p.n_tiles = (int)((N + lin::BM - 1) / lin::BM);
  p.kc = (int)((K + lin::BK - 1) / lin::BK);
  const int sp = (int)linear_s_pad(S);
  const bool bf = dtype == LSB_DTYPE_BF16;
  LinKern kern = bf ? pick_kernel<1>(sp) : pick_kernel<0>(sp);
  const int smem_max = (lin::SMEM_BUDGET / 1024 + 2) * 1024;  // every layout fits under it
  static SmemLimit smem_limit[8];
  if (int e = smem_limit[(bf ? 4 : 0) + sp / 32 - 1].ensure(kern, smem_max, "linear smem attribute"))
    return e;

  // Split and cluster count: the per-CTA critical path is
  //   ceil(tiles / clusters) * (ceil(kc / split) + overhead(split))
  // chunks; take the split that minimises it (ties: the smaller split).
  const int sms = num_sms();
  int best_split = 1, best_clusters = 1;
  double best_cost = 1e30;
  for (int s = 1; s <= lin::MAX_SPLIT && s <= p.kc; ++s) {
    int mc = 0;
    if (int e = max_clusters(kern, smem_max, s, &mc)) return e;
    if (mc <= 0) continue;
    const int clusters = std::min({mc, sms / s, p.n_tiles});
    if (clusters <= 0) continue;
    const int rounds = (p.n_tiles + clusters - 1) / clusters;
    const double cost = rounds * ((double)((p.kc + s - 1) / s) + (s > 1 ? 1.5 : 0.5));
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best_split = s;
      best_clusters = clusters;
    }
  }
  p.split = best_split;
  p.clusters = best_clusters;
  const int smem = linear_layout(sp, p.split, &p);

  CUtensorMap mx;
  const int64_t sx[4] = {0, 0, ldx, 1};
  if (int rc = make_bhnd_map(&mx, x, dtype, 1, 1, S, K, sx, lin::BK, (uint32_t)sp)) return rc;
  p.w_packed = static_cast<const uint8_t*>(w_packed);

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.clusters * p.split));
  cfg.blockDim = dim3(lin::THREADS);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)p.split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  LSB_CUDA_OK(cudaLaunchKernelEx(&cfg, kern, mx, p), "linear launch");
  LSB_CHECK_LAUNCH("linear");
  return LSB_OK;
}

namespace lsb {
int linear_device_error(bool reset) { return sm100::tu_device_error(reset); }
}  // namespace lsb
