// Input stage of the triangle multiplicative update (sm_100a).
//
// Reference work replaced (fast_trimul/_kernels.py:520-524 plus the permute copies
// of :138-139 / :155-156):   z_n = LayerNorm(z*mask);  a = (z_n W_ap + b_ap) *
// sigmoid(z_n W_ag + b_ag);  b likewise;  a, b written channel-major.
//
// One persistent CTA per SM. Per tile of 128 positions:
//   warp 0      TMA: z tile (2 x 16 KB, 128B-swizzled, K-major) into a ring slot;
//               the folded weight W' = [W_ap;W_ag;W_bp;W_bg]*diag(gamma_in) (512 x 128
//               fp16, 128 KB) is loaded once and stays resident.
//   warps 2-9   per row (two threads per row): fp32 mean/variance of z*mask, then the normalised row
//               LN(z*mask) (without gamma/beta, which are folded into W') written
//               back in place as fp16 -- the tensor cores' B operand.
//   warp 1      one thread issues tcgen05.mma with the WEIGHT as the A operand and the
//               z tile as B (M = 128 channels, N = 128 positions, K = 16) so TMEM lanes
//               are channels and columns are positions: slot 0 = [a_p | a_g], slot 1 =
//               [b_p | b_g], 256 columns each.
//   warps 10-17 TMEM -> registers (lane = channel, 32 positions per load);
//               proj = acc + (W beta + b), a = proj_p * sigmoid(proj_g); each warp stages a [32 channel x 32
//               position] block in shared memory and TMA-stores it into the channel
//               planes a_cm[b][c][u][v] -- or, row-sharded over P GPUs, straight into
//               the receive planes of the ranks that own each channel group (one
//               tensor map per destination, peer memory over NVLink).
// The two TMEM slots are independent, so the MMA of tile t+1's a-slot overlaps the
// epilogue of tile t's b-slot.
#include "ftm_kernels.h"

namespace ftm {

namespace {

constexpr int kZTile = 128 * kC * 2;          // 32 KB fp16 z tile
constexpr int kXformWarps = 8;
constexpr int kWBytes = 4 * kC * kC * 2;      // 128 KB
constexpr int kOffW = 0;
constexpr int kOffZ = kOffW + kWBytes;
constexpr int kStageBytes = 32 * 64 * 2;       // one warp's 32 channels x 64 positions
constexpr int kOffStage = kOffZ + kInBufs * kZTile;
constexpr int kOffBar = kOffStage + 8 * kStageBytes;
constexpr int kNumBars = 1 + 3 * kInBufs + 4 + 1;
constexpr int kOffTmem = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmem + 16 + 1024;  // + alignment slack

__global__ void __launch_bounds__(kInThreads, 1)
input_stage_kernel(const __grid_constant__ CUtensorMap zmap,
                   const __grid_constant__ CUtensorMap wmap,
                   const __grid_constant__ StoreMaps smaps, const float* __restrict__ mask,
                   const float* __restrict__ /*u_in: unused, rows are pre-normalised*/,
                   const float* __restrict__ v_in,
                   float2* __restrict__ zstats, PosTiling tl, int incoming, int z_bf16, float eps,
                   int* err, int test_stall) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sW = smem + kOffW;
  uint8_t* sZ = smem + kOffZ;
  uint8_t* sStage = smem + kOffStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* w_full = bars;
  uint64_t* z_full = bars + 1;
  uint64_t* a_ready = z_full + kInBufs;
  uint64_t* buf_empty = a_ready + kInBufs;
  uint64_t* tmem_full = buf_empty + kInBufs;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* mma_drain = tmem_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(w_full, 1);
    for (int s = 0; s < kInBufs; ++s) {
      mbar_init(&z_full[s], 1);
      mbar_init(&a_ready[s], 32 * kXformWarps);
      mbar_init(&buf_empty[s], 1);  // MMA commit: the tile was read by the tensor cores
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&tmem_full[h], 1);
      mbar_init(&tmem_empty[h], 8);
    }
    mbar_init(mma_drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  grid_dep_wait();      // z, mask, weights and the buffers this stage writes are free now
  grid_dep_release();

  const int ntiles = tl.tiles;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&zmap);
      tma_prefetch_desc(&wmap);
      mbar_arrive_expect_tx(w_full, kWBytes);
      for (int kc = 0; kc < 2; ++kc)
        for (int h = 0; h < 2; ++h)
          tma_load_2d(&wmap, w_full, sW + kc * 65536 + h * 32768, kc * 64, h * 256);
      int it = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
        const int s = it % kInBufs;
        const uint32_t ph = (it / kInBufs) & 1;
        for (int d = (it == 0 ? 1 : max(tl.pf, 1)); d <= tl.pf; ++d) {   // keep tl.pf tiles ahead in L2
          const int tp = t + d * static_cast<int>(gridDim.x);
          if (tp < ntiles) {
            int pb, pu, pv;
            tl.tile(tp, pb, pu, pv);
            tma_prefetch_l2_4d(&zmap, 0, pv, pu, pb);
            tma_prefetch_l2_4d(&zmap, 64, pv, pu, pb);
          }
        }
        if (!mbar_wait(&buf_empty[s], ph ^ 1, err, err_code(KERNEL_INPUT, ROLE_PRODUCER, 1))) break;
        // failure-detection test: CTA 0 never loads its first tile, so the waits on it
        // must expire, record the error and let every role drain and exit
        if (test_stall && blockIdx.x == 0) break;
        int b, u0, v0;
        tl.tile(t, b, u0, v0);
        uint8_t* dst = sZ + s * kZTile;
        mbar_arrive_expect_tx(&z_full[s], kZTile);
        tma_load_4d(&zmap, &z_full[s], dst, 0, v0, u0, b);
        tma_load_4d(&zmap, &z_full[s], dst + kZTile / 2, 64, v0, u0, b);
      }
      // copies still in flight must land before the CTA exits
      for (int i = (it > kInBufs ? it - kInBufs : 0); i < it; ++i)
        mbar_wait_drain(&z_full[i % kInBufs], (i / kInBufs) & 1);
      mbar_wait_drain(w_full, 0);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(0, 128, 128, 0, 0);
      const uint32_t wbase = smem_u32(sW);
      const uint32_t zbase = smem_u32(sZ);
      bool ok = mbar_wait(w_full, 0, err, err_code(KERNEL_INPUT, ROLE_MMA, 1));
      tc_fence_after();
      int it = 0;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x, ++it) {
        const int s = it % kInBufs;
        if (!mbar_wait(&a_ready[s], (it / kInBufs) & 1, err, err_code(KERNEL_INPUT, ROLE_MMA, 2))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t zb = zbase + s * kZTile;
        for (int h = 0; h < 2; ++h) {
          if (!mbar_wait(&tmem_empty[h], (it & 1) ^ 1, err, err_code(KERNEL_INPUT, ROLE_MMA, 3))) {
            ok = false;
            break;
          }
          tc_fence_after();
          // D[channel][position] = W'[2h+g] (128 ch x 128 k) * z^T; g = 0 proj, 1 gate
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            const uint32_t d = tmem_base + h * 256 + g * 128;
            const uint32_t wg = wbase + (2 * h + g) * 16384;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint64_t ad = kmajor_desc(wg + (kk >> 2) * 65536 + (kk & 3) * 32);
              const uint64_t bd = kmajor_desc(zb + (kk >> 2) * (kZTile / 2) + (kk & 3) * 32);
              umma_f16(d, ad, bd, idesc, kk > 0 ? 1u : 0u);
            }
          }
          umma_commit(&tmem_full[h]);
        }
        if (!ok) break;
        umma_commit(&buf_empty[s]);
      }
      // make sure every MMA this thread issued has finished before TMEM is freed
      umma_commit(mma_drain);
      mbar_wait_drain(mma_drain, 0);
    }
  } else if (warp < 2 + kXformWarps) {
    // ------------------------------------------------- LayerNorm of each row
    // lanes l and l^16 of a warp share one row, each owning one 64-channel half
    // (one 128-byte swizzled K chunk); partial sums are combined by shuffle
    const int tw = warp - 2;
    const int row = tw * 16 + (lane & 15);
    const int half = lane >> 4;
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const int s = it % kInBufs;
      int b, u0, v0;
      tl.tile(t, b, u0, v0);
      const int u = u0 + row / tl.vt, v = v0 + row % tl.vt;
      const bool valid = (u < tl.R) && (v < tl.S);
      // the mask load is issued before the wait so its latency hides behind the TMA
      // position of this row in z's natural (b, r, s) order
      // (incoming: the tiling runs over u = z column, v = z row, so z is (tl.S x tl.R))
      const size_t zi = incoming ? (static_cast<size_t>(b) * tl.S + v) * tl.R + u
                                 : (static_cast<size_t>(b) * tl.R + u) * tl.S + v;
      float m = 0.f;
      if (valid) m = mask ? __ldg(mask + zi) : 1.f;
      if (!mbar_wait(&z_full[s], (it / kInBufs) & 1, err, err_code(KERNEL_INPUT, ROLE_TRANSFORM, 1)))
        break;
      uint8_t* zt = sZ + s * kZTile + half * (kZTile / 2);
      uint4 raw[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) raw[q] = *reinterpret_cast<const uint4*>(zt + sw128_off(row, q));
      // two-pass LayerNorm statistics in fp32, then the normalised row
      // LN(m*z) = m*rstd*(z - mean) (rstd = 1/sqrt(m^2 var + eps)) written back in
      // place as fp16: the operand the tensor cores read (gamma/beta are folded into
      // W' and v at pack time). Eight independent partial sums per thread.
      float f[64];                         // this thread's 64 values, unpacked once
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float t8[8];
        unpack8(raw[q], z_bf16, t8);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[q * 8 + e] = t8[e];
      }
      // packed fp32x2 arithmetic (FADD2 / FFMA2): eight partial sums in four pairs
      float2 ps[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) ps[e] = make_float2(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < 32; ++i) ps[i & 3] = __fadd2_rn(ps[i & 3], make_float2(f[2 * i], f[2 * i + 1]));
      float tot = ((ps[0].x + ps[0].y) + (ps[1].x + ps[1].y)) + ((ps[2].x + ps[2].y) + (ps[3].x + ps[3].y));
      tot += __shfl_xor_sync(0xffffffffu, tot, 16);
      const float mean = tot * (1.0f / kC);
      const float2 nmean = make_float2(-mean, -mean);
#pragma unroll
      for (int e = 0; e < 4; ++e) ps[e] = make_float2(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float2 d = __fadd2_rn(make_float2(f[2 * i], f[2 * i + 1]), nmean);
        ps[i & 3] = __ffma2_rn(d, d, ps[i & 3]);
      }
      float sq = ((ps[0].x + ps[0].y) + (ps[1].x + ps[1].y)) + ((ps[2].x + ps[2].y) + (ps[3].x + ps[3].y));
      sq += __shfl_xor_sync(0xffffffffu, sq, 16);
      const float var = sq * (1.0f / kC);
      const float sa = m * rsqrtf(m * m * var + eps);
      const float sb = -mean * sa;
      if (valid && half == 0) zstats[zi] = make_float2(mean, sa);   // reused by the output stage
      const float2 sa2 = make_float2(sa, sa), sb2 = make_float2(sb, sb);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 y = __ffma2_rn(make_float2(f[q * 8 + 2 * e], f[q * 8 + 2 * e + 1]), sa2, sb2);
          o[e] = pack_half2(y.x, y.y);
        }
        *reinterpret_cast<uint4*>(zt + sw128_off(row, q)) = make_uint4(o[0], o[1], o[2], o[3]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&a_ready[s]);
    }
  } else {
    // ----------------------------------------------------------------- epilogue
    // warp -> (TMEM lane quarter = 32 channels, half of the tile's 128 positions)
    const int ew = warp - 2 - kXformWarps;
    const int quarter = warp & 3;
    const int phalf = ew >> 2;
    const int c = quarter * 32 + lane;                 // this thread's channel
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    float vp[2], vg[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      // halves of the biases: a = h_p (1 + tanh(h_g)) with h_p = (acc_p + v_p) / 2,
      // h_g = (acc_g + v_g) / 2 -- the logistic gate in its tanh form
      vp[h] = 0.5f * __ldg(v_in + h * 256 + c);
      vg[h] = 0.5f * __ldg(v_in + h * 256 + 128 + c);
    }
    uint8_t* stage = sStage + ew * kStageBytes;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x, ++it) {
      int b, u0, v0;
      tl.tile(t, b, u0, v0);
      for (int h = 0; h < 2; ++h) {
        if (!mbar_wait_warp(&tmem_full[h], it & 1, err, err_code(KERNEL_INPUT, ROLE_EPILOGUE, 2))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const CUtensorMap* omaps = h == 0 ? smaps.a : smaps.b;
        // the previous store from this warp's staging buffer must have read it
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
#pragma unroll 1
        for (int j = 0; j < 2; ++j) {
          const int p0 = phalf * 64 + j * 32;        // first tile row of this chunk
          float p[32], g[32];
          tmem_ld32x2(lane_base + h * 256 + p0, lane_base + h * 256 + 128 + p0, p, g);
          uint32_t packed[16];
          const float2 half2f = make_float2(0.5f, 0.5f);
          const float2 vp2 = make_float2(vp[h], vp[h]), vg2 = make_float2(vg[h], vg[h]);
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float2 a2 = gated_tanh_half2(__ffma2_rn(half2f, make_float2(p[i], p[i + 1]), vp2),
                                               __ffma2_rn(half2f, make_float2(g[i], g[i + 1]), vg2));
            packed[i / 2] = pack_half2(a2.x, a2.y);
          }
          // staging row = channel, 64 positions (128 B, 128-byte swizzle)
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(stage + sw128_off(lane, j * 4 + q)) =
                make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        {
          const int p0 = phalf * 64;
          const int u = u0 + p0 / tl.vt, v = v0 + p0 % tl.vt;
          if (lane == 0 && u < tl.R && v < tl.S) {
            // this warp's 32 channels; a destination map holds smaps.lq channels (one
            // map unless the channels are scattered to their owner ranks)
            for (int s2 = 0; s2 < 32; s2 += smaps.box_c) {
              const int c = quarter * 32 + s2, q = c / smaps.lq;
              tma_store_4d(omaps + q, stage + s2 * 128, v, u, c - q * smaps.lq, smaps.blk_base + b);
            }
            bulk_commit();
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tmem_empty[h]);
      }
      __syncwarp();
    }
    if (lane == 0) bulk_wait0();  // stores complete before the kernel ends
    if (smaps.sys_fence) __threadfence_system();   // peers' planes: visible to their owners
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace

size_t input_stage_smem_bytes() { return kSmemBytes; }

cudaError_t launch_input_stage(const CUtensorMap& zmap, const CUtensorMap& wmap,
                               const StoreMaps& smaps, const float* mask,
                               const float* u_in, const float* v_in, float2* zstats,
                               const PosTiling& tl, int incoming, int z_bf16, float eps, int* err,
                               int grid, cudaStream_t stream, int test_stall) {
  cudaError_t e = set_smem_once(reinterpret_cast<const void*>(input_stage_kernel), kSmemBytes);
  if (e != cudaSuccess) return e;
  return launch_pdl(input_stage_kernel, dim3(grid), dim3(kInThreads), kSmemBytes, stream, nullptr, 0,
                    zmap, wmap, smaps, mask, u_in, v_in, zstats, tl, incoming, z_bf16, eps, err,
                    test_stall);
}

}  // namespace ftm
