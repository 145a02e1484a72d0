// Triangle contraction (sm_100a): X[l][i][j] = sum_k A[l][i][k] * B[l][j][k].
//
// Reference work replaced: outgoing()/incoming() (fast_trimul/_kernels.py:131-162),
// a CuTe-DSL Ampere mma.sync batched GEMM fed by permute copies. Here both operands
// arrive K-major from the input stage (incoming mode is handled by the input stage
// writing the transposed layout), so one kernel serves both modes.
//
// Persistent, one CTA per SM, warp-specialised:
//   warp 0     TMA producer: 4-stage ring of {A 128x64, B 256x64} fp16 tiles
//              (128B swizzle, plain per-CTA loads -- no cluster multicast).
//   warp 1     one thread issues tcgen05.mma M=128 N=256 K=16 into a TMEM
//              accumulator; two accumulators (2 x 256 columns) alternate between
//              tiles so the epilogue of tile t overlaps the mainloop of tile t+1.
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time, fp32 -> fp16, 16-byte stores.
// Tiles are visited channel (l) major so the CTAs working at the same time share
// one channel's A and B in L2.
#include "ftm_kernels.h"

namespace ftm {

namespace {

constexpr int kATile = kCtBM * kCtBK * 2;  // 16 KB
constexpr int kBTile = kCtBN * kCtBK * 2;  // 32 KB
constexpr int kStageBytes = kATile + kBTile;
constexpr int kOffBar = kCtStages * kStageBytes;
constexpr int kNumBars = 2 * kCtStages + 4 + 1;
constexpr int kOffTmem = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmem + 16 + 1024;

__global__ void __launch_bounds__(kCtThreads, 1)
contraction_kernel(const __grid_constant__ CUtensorMap amap,
                   const __grid_constant__ CUtensorMap bmap, __half* __restrict__ X, int L,
                   int M, int N, int K, int rows_per_block, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + kCtStages;
  uint64_t* tmem_full = bars + 2 * kCtStages;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* mma_drain = tmem_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kCtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 4);
    }
    mbar_init(mma_drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles_m = (M + kCtBM - 1) / kCtBM;
  const int tiles_n = (N + kCtBN - 1) / kCtBN;
  const int per_l = tiles_m * tiles_n;
  const int ntiles = L * per_l;
  const int nk = (K + kCtBK - 1) / kCtBK;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&amap);
      tma_prefetch_desc(&bmap);
      int st = 0;
      uint32_t ph = 0;
      long issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
        const int l = t / per_l;
        const int r = t - l * per_l;
        const int tm = r / tiles_n, tn = r - (r / tiles_n) * tiles_n;
        const int j0 = tn * kCtBN;
        const int blk = j0 / rows_per_block, jl = j0 - blk * rows_per_block;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[st], ph ^ 1, err, err_code(KERNEL_CONTRACT, ROLE_PRODUCER, 1))) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + st * kStageBytes;
          mbar_arrive_expect_tx(&full[st], kStageBytes);
          tma_load_3d(&amap, &full[st], sa, kb * kCtBK, tm * kCtBM, l);
          tma_load_4d(&bmap, &full[st], sa + kATile, kb * kCtBK, jl, l, blk);
          ++issued;
          if (++st == kCtStages) {
            st = 0;
            ph ^= 1;
          }
        }
      }
      // drain: the last min(issued, stages) loads must land before exit
      const long first = issued > kCtStages ? issued - kCtStages : 0;
      for (long i = first; i < issued; ++i)
        mbar_wait_drain(&full[i % kCtStages], static_cast<uint32_t>((i / kCtStages) & 1));
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(0, kCtBM, kCtBN, 0, 0);
      const uint32_t base = smem_u32(smem);
      int st = 0;
      uint32_t ph = 0;
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x, ++it) {
        const int acc = it & 1;
        if (!mbar_wait(&tmem_empty[acc], ((it >> 1) & 1) ^ 1, err,
                       err_code(KERNEL_CONTRACT, ROLE_MMA, 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * kCtBN;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[st], ph, err, err_code(KERNEL_CONTRACT, ROLE_MMA, 2))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + st * kStageBytes;
#pragma unroll
          for (int kk = 0; kk < kCtBK / 16; ++kk) {
            const uint64_t ad = kmajor_desc(sa + kk * 32);
            const uint64_t bd = kmajor_desc(sa + kATile + kk * 32);
            umma_f16(d, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[st]);
          if (++st == kCtStages) {
            st = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tmem_full[acc]);
      }
      umma_commit(mma_drain);
      mbar_wait_drain(mma_drain, 0);
    }
  } else {
    const int sub = warp & 3;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(sub * 32) << 16);
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const int l = t / per_l;
      const int r = t - l * per_l;
      const int tm = r / tiles_n, tn = r - (r / tiles_n) * tiles_n;
      if (!mbar_wait_warp(&tmem_full[acc], (it >> 1) & 1, err, err_code(KERNEL_CONTRACT, ROLE_EPILOGUE, 1)))
        break;
      tc_fence_after();
      const int i = tm * kCtBM + sub * 32 + lane;
      __half* xrow = X + (static_cast<size_t>(l) * M + i) * N;
#pragma unroll 1
      for (int ch = 0; ch < kCtBN / 32; ++ch) {
        float v[32];
        tmem_ld32(lane_base + acc * kCtBN + ch * 32, v);
        const int j = tn * kCtBN + ch * 32;
        if (i < M) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (j + q * 8 < N) {
              uint4 o;
              o.x = pack_half2(v[q * 8 + 0], v[q * 8 + 1]);
              o.y = pack_half2(v[q * 8 + 2], v[q * 8 + 3]);
              o.z = pack_half2(v[q * 8 + 4], v[q * 8 + 5]);
              o.w = pack_half2(v[q * 8 + 6], v[q * 8 + 7]);
              *reinterpret_cast<uint4*>(xrow + j + q * 8) = o;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace

size_t contraction_smem_bytes() { return kSmemBytes; }

cudaError_t launch_contraction(const CUtensorMap& amap, const CUtensorMap& bmap, __half* X, int L,
                               int M, int N, int K, int rows_per_block, int* err, int grid,
                               cudaStream_t stream) {
  cudaError_t e = set_smem_once(reinterpret_cast<const void*>(contraction_kernel), kSmemBytes);
  if (e != cudaSuccess) return e;
  contraction_kernel<<<grid, kCtThreads, kSmemBytes, stream>>>(amap, bmap, X, L, M, N, K,
                                                               rows_per_block, err);
  return cudaGetLastError();
}

}  // namespace ftm
