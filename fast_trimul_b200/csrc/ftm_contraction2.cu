// Triangle contraction on CTA pairs (sm_100a, tcgen05.mma.cta_group::2).
//
// Same operation as ftm_contraction.cu, X[l][i][j] = sum_k A[l][i][k] * B[l][j][k]
// (replacing outgoing()/incoming(), fast_trimul/_kernels.py:131-162), with a
// 256 x 256 output tile computed by two CTAs of a cluster that share one MMA:
//   * each CTA TMA-loads only its own halves -- A rows [128 r, 128 r + 128) and
//     B rows [128 r, 128 r + 128) of the tile -- into a 6-stage ring (32 KB/stage);
//     the transfers of both CTAs complete on the leader CTA's full barrier
//     (.cta_group::2 completion). No cluster multicast is used anywhere.
//     A (with X) and B may each be stored as row blocks -- the layouts that NCCL
//     all-gathers / all-to-alls between row shards and channel shards produce.
//   * the leader's MMA thread issues M=256 N=256 K=16 MMAs reading A and B from
//     both CTAs' shared memory; each CTA's TMEM receives its 128 rows.
//   * stage release and accumulator-ready notifications reach the peer CTA by a
//     second tcgen05.commit aimed at the peer's barrier (shared::cluster address);
//     the peer's epilogue warps signal the leader's accumulator-empty barrier with
//     remote mbarrier arrives.
// Per CTA this halves the L2->SM operand traffic per FLOP of the single-CTA
// 128 x 256 tile (64 instead of 96 bytes per MMA clock) and doubles the stage depth.
#include "ftm_kernels.h"

namespace ftm {

namespace {

constexpr int kBM = 128, kBN = 128, kBK = 64;   // per-CTA halves of one 256 x 256 MMA tile
constexpr int kATile = kBM * kBK * 2;          // 16 KB
constexpr int kBTile = kBN * kBK * 2;          // 16 KB
constexpr int kThreads = 192;

// NH = number of 256-wide N halves per pair tile: NH = 1 gives 256 x 256 tiles with two
// 256-column TMEM accumulators (the epilogue of one tile overlaps the next tile's MMAs);
// NH = 2 gives 256 x 512 tiles whose two N halves share each A stage (a third less
// operand traffic per FLOP from L2) in one 512-column accumulator.
template <int NH>
struct PairCfg {
  static constexpr int kStages = NH == 1 ? 6 : 4;
  static constexpr int kStageBytes = kATile + NH * kBTile;
  static constexpr int kAcc = NH == 1 ? 2 : 1;          // accumulators in TMEM
  static constexpr int kAccCols = 256 * NH;             // columns per accumulator
  static constexpr int kOffBar = kStages * kStageBytes;
  static constexpr int kNumBars = 2 * kStages + 2 * kAcc + 1;
  static constexpr int kOffTmem = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffTmem + 16 + 1024;
  static_assert(kSmemBytes <= 232448, "pair contraction exceeds 227 KB of shared memory");
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t num_clusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// shared::cluster address of `p` (a local shared-memory object) in CTA `rank`
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void remote_arrive(uint32_t cl_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cl_addr)
               : "memory");
}
// operand tiles: (k within its k block, row within its row block, l, row block, k block)
__device__ __forceinline__ void tma_load_5d_pair(const CUtensorMap* map, uint32_t bar_cl, void* dst,
                                                 int c0, int c1, int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar_cl), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on the barrier at shared::cluster address `cl` (this CTA or the peer) once
// all previously issued pair MMAs have completed
__device__ __forceinline__ void umma_commit_pair(uint32_t cl) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cl)
               : "memory");
}

// AMN / BMN: operand A / B is MN-major (its rows contiguous in memory, k strided), loaded
// as two 64-row swizzled atoms per 128-row half; the backward's transposed products
// (dA = dX B, dB = dX^T A) read their operands this way without a transpose pass.
template <int NH, int AMN = 0, int BMN = 0>
__global__ void __launch_bounds__(kThreads, 1)
contraction_pair_kernel(const __grid_constant__ CUtensorMap amap,
                        const __grid_constant__ CUtensorMap bmap, __half* __restrict__ X, int L,
                        int M, int N, int K, const CtLayout lay, int* err, const XDest xd) {
  using Cfg = PairCfg<NH>;
  constexpr int kStages = Cfg::kStages, kStageBytes = Cfg::kStageBytes, kAcc = Cfg::kAcc;
  constexpr int kAccCols = Cfg::kAccCols;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* full = bars;                  // leader: operands of both CTAs landed
  uint64_t* empty = bars + kStages;       // both: stage consumed by the pair MMA
  uint64_t* tmem_full = bars + 2 * kStages;
  uint64_t* tmem_empty = tmem_full + kAcc;   // leader: 4 local + 4 peer epilogue warps
  uint64_t* mma_drain = tmem_empty + kAcc;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kOffTmem);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < kAcc; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 8);
    }
    mbar_init(mma_drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  grid_dep_wait();     // operands written, X free
  grid_dep_release();

  const int tiles_m = (M + 2 * kBM - 1) / (2 * kBM);
  const int tiles_n = (N + 2 * kBN * NH - 1) / (2 * kBN * NH);
  const int per_l = tiles_m * tiles_n;
  const int ntiles = L * per_l;
  const int nk = (K + kBK - 1) / kBK;
  const int cid = static_cast<int>(cluster_id_x());
  const int ncl = static_cast<int>(num_clusters_x());

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer (both CTAs)
      tma_prefetch_desc(&amap);
      tma_prefetch_desc(&bmap);
      int st = 0;
      uint32_t ph = 0;
      long issued = 0;
      bool ok = true;
      for (int t = cid; ok && t < ntiles; t += ncl) {
        const int l = t / per_l;
        const int r = t - l * per_l;
        const int tm = r / tiles_n, tn = r - (r / tiles_n) * tiles_n;
        const int i0 = tm * 2 * kBM + static_cast<int>(rank) * kBM;
        const int ablk = i0 / lay.a_rpb, ail = i0 - ablk * lay.a_rpb;
        int bblk[NH], bjl[NH];
#pragma unroll
        for (int h = 0; h < NH; ++h) {
          const int j0 = (tn * NH + h) * 2 * kBN + static_cast<int>(rank) * kBN;
          bblk[h] = j0 / lay.b_rpb;
          bjl[h] = j0 - bblk[h] * lay.b_rpb;
        }
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[st], ph ^ 1, err, err_code(KERNEL_CONTRACT, ROLE_PRODUCER, 2))) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + st * kStageBytes;
          const uint32_t fb = cluster_addr(&full[st], 0);
          if (leader) mbar_arrive_expect_tx(&full[st], 2 * kStageBytes);
          // rows of A / B may be split into row blocks and k into k blocks (each 64-wide
          // k step lies inside one k block): 5-D coordinates
          // (k in block, row in block, l, row block, k block)
          const int kg = kb * kBK;
          const int kblk = kg / lay.k_rpb;
          const int kc = kg - kblk * lay.k_rpb;
          if (AMN) {
            tma_load_5d_pair(&amap, fb, sa, i0, kg, l, 0, 0);
            tma_load_5d_pair(&amap, fb, sa + kATile / 2, i0 + 64, kg, l, 0, 0);
          } else {
            tma_load_5d_pair(&amap, fb, sa, kc, ail, l, ablk, kblk);
          }
#pragma unroll
          for (int h = 0; h < NH; ++h) {
            uint8_t* sb = sa + kATile + h * kBTile;
            if (BMN) {
              const int j0 = (tn * NH + h) * 2 * kBN + static_cast<int>(rank) * kBN;
              tma_load_5d_pair(&bmap, fb, sb, j0, kg, l, 0, 0);
              tma_load_5d_pair(&bmap, fb, sb + kBTile / 2, j0 + 64, kg, l, 0, 0);
            } else {
              tma_load_5d_pair(&bmap, fb, sb, kc, bjl[h], l, bblk[h], kblk);
            }
          }
          ++issued;
          if (++st == kStages) {
            st = 0;
            ph ^= 1;
          }
        }
      }
      if (leader) {
        const long first = issued > kStages ? issued - kStages : 0;
        for (long i = first; i < issued; ++i)
          mbar_wait_drain(&full[i % kStages], static_cast<uint32_t>((i / kStages) & 1));
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      // ------------------------------------------------ pair MMA issuer (leader)
      constexpr uint32_t idesc = idesc_f16(0, 2 * kBM, 2 * kBN, AMN, BMN);
      const uint32_t base = smem_u32(smem);
      int st = 0;
      uint32_t ph = 0;
      int it = 0;
      bool ok = true;
      for (int t = cid; ok && t < ntiles; t += ncl, ++it) {
        const int acc = it % kAcc;
        if (!mbar_wait(&tmem_empty[acc], ((it / kAcc) & 1) ^ 1, err,
                       err_code(KERNEL_CONTRACT, ROLE_MMA, 4))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * kAccCols;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[st], ph, err, err_code(KERNEL_CONTRACT, ROLE_MMA, 5))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + st * kStageBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // K-major: 16 k = 32 bytes along a swizzled row; MN-major: 16 k = 16 rows of
            // two 64-element atoms 8 KB apart
            const uint64_t ad = AMN ? sw128_desc(sa + kk * 2048, kATile / 2, 1024) : kmajor_desc(sa + kk * 32);
#pragma unroll
            for (int h = 0; h < NH; ++h) {
              const uint32_t sb = sa + kATile + h * kBTile;
              const uint64_t bd = BMN ? sw128_desc(sb + kk * 2048, kBTile / 2, 1024) : kmajor_desc(sb + kk * 32);
              umma_f16_pair(d + h * 256, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
            }
          }
          umma_commit_pair(cluster_addr(&empty[st], 0));
          umma_commit_pair(cluster_addr(&empty[st], 1));
          if (++st == kStages) {
            st = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(cluster_addr(&tmem_full[acc], 0));
        umma_commit_pair(cluster_addr(&tmem_full[acc], 1));
      }
      umma_commit_pair(cluster_addr(mma_drain, 0));
      mbar_wait_drain(mma_drain, 0);
    }
  } else {
    // ------------------------------------------------ epilogue (both CTAs)
    const int sub = warp & 3;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(sub * 32) << 16);
    int it = 0;
    for (int t = cid; t < ntiles; t += ncl, ++it) {
      const int acc = it % kAcc;
      const int l = t / per_l;
      const int r = t - l * per_l;
      const int tm = r / tiles_n, tn = r - (r / tiles_n) * tiles_n;
      if (!mbar_wait_warp(&tmem_full[acc], (it / kAcc) & 1, err,
                          err_code(KERNEL_CONTRACT, ROLE_EPILOGUE, 2)))
        break;
      tc_fence_after();
      const int i = tm * 2 * kBM + static_cast<int>(rank) * kBM + sub * 32 + lane;
      // X rows are stored in row blocks with the strides of `lay`, or -- scattered --
      // each block straight into its owner's channel-major plane
      const int xb = i / lay.x_rpb, xi = i - xb * lay.x_rpb;
      __half* xrow =
          xd.enabled
              ? xd.base[xb] + ((static_cast<size_t>(l / xd.lq) * xd.c_total + xd.chan_off + l % xd.lq) *
                                   lay.x_rpb + xi) * N
              : X + xb * lay.x_bs + l * lay.x_ls + xi * lay.x_rs;
      // 16-column chunks, the TMEM load of chunk ch + 1 in flight while chunk ch is
      // converted and stored
      uint32_t va[2][16];
      tmem_ld16_nowait(lane_base + acc * kAccCols, va[0]);
      tmem_wait_ld();
#pragma unroll
      for (int ch = 0; ch < kAccCols / 16; ++ch) {
        const int cur = ch & 1;
        if (ch + 1 < kAccCols / 16) tmem_ld16_nowait(lane_base + acc * kAccCols + (ch + 1) * 16, va[cur ^ 1]);
        const int j = tn * kAccCols + ch * 16;
        if (i < M) {
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            if (j + q * 8 < N) {
              uint4 o;
              o.x = pack_half2(__uint_as_float(va[cur][q * 8 + 0]), __uint_as_float(va[cur][q * 8 + 1]));
              o.y = pack_half2(__uint_as_float(va[cur][q * 8 + 2]), __uint_as_float(va[cur][q * 8 + 3]));
              o.z = pack_half2(__uint_as_float(va[cur][q * 8 + 4]), __uint_as_float(va[cur][q * 8 + 5]));
              o.w = pack_half2(__uint_as_float(va[cur][q * 8 + 6]), __uint_as_float(va[cur][q * 8 + 7]));
              *reinterpret_cast<uint4*>(xrow + j + q * 8) = o;
            }
          }
        }
        if (ch + 1 < kAccCols / 16) tmem_wait_ld();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&tmem_empty[acc]);
        else remote_arrive(cluster_addr(&tmem_empty[acc], 0));
      }
    }
    if (xd.enabled) __threadfence_system();   // rows stored into peers' planes
  }

  // After a failure the two CTAs may have issued different numbers of loads, and the
  // leader's drain only covers its own: give any copy still landing in this CTA's
  // shared memory time to finish (bounded, error path only) before leaving.
  if (grid_failed(err)) {
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 200000ull) __nanosleep(1000);
  }
  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still touch its memory
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(512)
                 : "memory");
  }
}

}  // namespace

cudaError_t launch_contraction_pair(const CUtensorMap& amap, const CUtensorMap& bmap, __half* X,
                                    int L, int M, int N, int K, const CtLayout& lay, int* err,
                                    int num_sms, cudaStream_t stream, const XDest* xdest,
                                    int a_mn, int b_mn) {
  XDest xd{};
  if (xdest) xd = *xdest;
  // FTM_CT_NH=2 selects the 256 x 512 tile variant
  const char* nh_env = getenv("FTM_CT_NH");
  const int nh = (nh_env && atoi(nh_env) == 2) ? 2 : 1;
  auto go = [&](auto kern, int smem_bytes, int tile_n) -> cudaError_t {
    cudaError_t e = set_smem_once(reinterpret_cast<const void*>(kern), smem_bytes);
    if (e != cudaSuccess) return e;
    const long tiles = long(L) * ((M + 255) / 256) * ((N + tile_n - 1) / tile_n);
    const int clusters = static_cast<int>(tiles < num_sms / 2 ? tiles : num_sms / 2);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    return launch_pdl(kern, dim3(2 * clusters), dim3(kThreads), smem_bytes, stream, attr, 1, amap,
                      bmap, X, L, M, N, K, lay, err, xd);
  };
  if (a_mn || b_mn) {
    if (a_mn && b_mn) return go(contraction_pair_kernel<1, 1, 1>, PairCfg<1>::kSmemBytes, 256);
    if (a_mn) return go(contraction_pair_kernel<1, 1, 0>, PairCfg<1>::kSmemBytes, 256);
    return go(contraction_pair_kernel<1, 0, 1>, PairCfg<1>::kSmemBytes, 256);
  }
  if (nh == 2) return go(contraction_pair_kernel<2>, PairCfg<2>::kSmemBytes, 512);
  return go(contraction_pair_kernel<1>, PairCfg<1>::kSmemBytes, 256);
}

}  // namespace ftm
