// Output stage of the triangle multiplicative update (sm_100a).
//
// Reference work replaced (fast_trimul/_kernels.py:526-530 and the mask / cast glue
// of functional.py:24-26):
//   x_n = LayerNorm_ch(x);  g = sigmoid(LN_cz(z*mask) W_g + b_g);
//   delta = g * (x_n W_o + b_o);  out = ((residual ? z*mask : 0) + delta) * mask.
//
// One persistent CTA per SM, 128 positions per tile, two ring slots:
//   warp 0     TMA: z tile (K-major, 128B swizzle) and the x tile straight from the
//              channel-major x (MN-major operand: 64-position atoms x 128 channels),
//              plus the resident folded weights [W_g diag(gamma_in); W_o diag(gamma_out)].
//   warps 2-5  per row: LayerNorm statistics of x (fp32), bf16 -> fp16 of z in place
//              when needed; the statistics of z*mask come from the input stage
//              (zstats), which normalised the same rows.
//   warp 1     tcgen05.mma: TMEM[0:128) = z W_g'^T (K-major A), TMEM[128:256) =
//              x W_o'^T (MN-major A); two 256-column accumulators alternate tiles.
//   warps 6-13 epilogue (two warps per TMEM lane quarter, each owning half of the
//              128 output channels): fold the statistics back in, gate, residual,
//              mask; 16-bit outputs are written over the z slot in place and
//              TMA-stored (32 positions x 64 channels per warp), fp32 stored directly.
#include "ftm_kernels.h"

namespace ftm {

namespace {

constexpr int kHalfTile = 128 * 64 * 2;   // 16 KB
constexpr int kZTile = 2 * kHalfTile;     // 32 KB
constexpr int kXTile = 2 * kHalfTile;     // 32 KB
constexpr int kSlot = kZTile + kXTile;
constexpr int kWBytes = 2 * kC * kC * 2;  // 64 KB
constexpr int kOffW = 0;
constexpr int kOffSlots = kOffW + kWBytes;
constexpr int kOffStats = kOffSlots + kOutBufs * kSlot;
constexpr int kStatRing = 4;  // per-tile statistics outlive their ring slot's x half
constexpr int kOffMask = kOffStats + kStatRing * 128 * 16;
constexpr int kOffUV = kOffMask + kStatRing * 128 * 4;
constexpr int kOffBar = kOffUV + 4 * kC * 4;
constexpr int kNumBars = 1 + 5 * kOutBufs + 4 + 1;
constexpr int kOffTmem = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmem + 16 + 1024;

template <int OUT_DT>
__device__ __forceinline__ void store_out32(void* out, size_t elem, const float (&r)[32]) {
  if (OUT_DT == 0) {  // fp32
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(out) + elem);
#pragma unroll
    for (int q = 0; q < 8; ++q) p[q] = make_float4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
  } else {
    uint4* p = reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + elem);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 o;
      if (OUT_DT == 1) {
        o.x = pack_half2(r[8 * q + 0], r[8 * q + 1]);
        o.y = pack_half2(r[8 * q + 2], r[8 * q + 3]);
        o.z = pack_half2(r[8 * q + 4], r[8 * q + 5]);
        o.w = pack_half2(r[8 * q + 6], r[8 * q + 7]);
      } else {
        o.x = pack_bf162(r[8 * q + 0], r[8 * q + 1]);
        o.y = pack_bf162(r[8 * q + 2], r[8 * q + 3]);
        o.z = pack_bf162(r[8 * q + 4], r[8 * q + 5]);
        o.w = pack_bf162(r[8 * q + 6], r[8 * q + 7]);
      }
      p[q] = o;
    }
  }
}

template <int OUT_DT>
__global__ void __launch_bounds__(kOutThreads, 1)
output_stage_kernel(const __grid_constant__ CUtensorMap zmap,
                    const __grid_constant__ CUtensorMap xmap,
                    const __grid_constant__ CUtensorMap wmap,
                    const __grid_constant__ CUtensorMap omap, const float* __restrict__ mask,
                    const float2* __restrict__ zstats,
                    const float* __restrict__ u_g, const float* __restrict__ v_g,
                    const float* __restrict__ u_o, const float* __restrict__ v_o,
                    void* __restrict__ out, PosTiling tl, int residual, int z_bf16,
                    float /*eps_in: applied by the input stage's zstats*/, float eps_out,
                    int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sW = smem + kOffW;
  uint8_t* sSlots = smem + kOffSlots;
  float4* sStats = reinterpret_cast<float4*>(smem + kOffStats);
  float* sMask = reinterpret_cast<float*>(smem + kOffMask);
  // per channel pair (2k, 2k+1): {u_g/2 x2, v_g/2 x2}, {u_o x2, v_o x2} -- gate constants
  // halved for the tanh form, laid out as float2 pairs for the packed fp32x2 epilogue
  float4* sUV = reinterpret_cast<float4*>(smem + kOffUV);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* w_full = bars;
  uint64_t* full_x = bars + 1;           // x half of a ring slot landed
  uint64_t* full_z = full_x + kOutBufs;  // z half landed
  uint64_t* a_ready = full_z + kOutBufs;
  uint64_t* x_empty = a_ready + kOutBufs;  // x half read by the MMA
  uint64_t* z_empty = x_empty + kOutBufs;  // z half done with (epilogue stored out)
  uint64_t* tmem_full = z_empty + kOutBufs;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* mma_drain = tmem_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(w_full, 1);
    for (int s = 0; s < kOutBufs; ++s) {
      mbar_init(&full_x[s], 1);
      mbar_init(&full_z[s], 1);
      mbar_init(&a_ready[s], 128);
      mbar_init(&x_empty[s], 1);    // MMA commit
      mbar_init(&z_empty[s], 8);    // epilogue warps
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 8);
    }
    mbar_init(mma_drain, 1);
    fence_mbar_init();
  }
  grid_dep_wait();      // x, z statistics, weights and the output buffer are ready / free
  for (int k = threadIdx.x; k < kC / 2; k += blockDim.x) {
    sUV[2 * k] = make_float4(0.5f * u_g[2 * k], 0.5f * u_g[2 * k + 1], 0.5f * v_g[2 * k], 0.5f * v_g[2 * k + 1]);
    sUV[2 * k + 1] = make_float4(u_o[2 * k], u_o[2 * k + 1], v_o[2 * k], v_o[2 * k + 1]);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int ntiles = tl.tiles;
  grid_dep_release();

  if (warp == 0) {
    // two producer lanes: lane 0 refills x halves as soon as the MMA has read them,
    // lane 1 refills z halves once the epilogue has stored the tile written over them
    if (lane == 0) {
      tma_prefetch_desc(&xmap);
      tma_prefetch_desc(&wmap);
      mbar_arrive_expect_tx(w_full, kWBytes);
      for (int kc = 0; kc < 2; ++kc) tma_load_2d(&wmap, w_full, sW + kc * 32768, kc * 64, 0);
      int it = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
        const int s = it % kOutBufs;
        for (int d = (it == 0 ? 1 : max(tl.pf, 1)); d <= tl.pf; ++d) {   // keep tl.pf tiles ahead in L2
          const int tp = t + d * static_cast<int>(gridDim.x);
          if (tp < ntiles) {
            int pb, pu, pv;
            tl.tile(tp, pb, pu, pv);
            for (int h = 0; h < 2; ++h)
              tma_prefetch_l2_4d(&xmap, tl.vt == 128 ? pv + 64 * h : pv, tl.vt == 128 ? pu : pu + h, 0, pb);
          }
        }
        if (!mbar_wait(&x_empty[s], ((it / kOutBufs) & 1) ^ 1, err,
                       err_code(KERNEL_OUTPUT, ROLE_PRODUCER, 1)))
          break;
        int b, u0, v0;
        tl.tile(t, b, u0, v0);
        uint8_t* xs = sSlots + s * kSlot + kZTile;
        mbar_arrive_expect_tx(&full_x[s], kXTile);
        for (int h = 0; h < 2; ++h) {
          const int jj = tl.vt == 128 ? v0 + 64 * h : v0;
          const int ii = tl.vt == 128 ? u0 : u0 + h;
          tma_load_4d(&xmap, &full_x[s], xs + h * kHalfTile, jj, ii, 0, b);
        }
      }
      for (int i = (it > kOutBufs ? it - kOutBufs : 0); i < it; ++i)
        mbar_wait_drain(&full_x[i % kOutBufs], (i / kOutBufs) & 1);
      mbar_wait_drain(w_full, 0);
    } else if (lane == 1) {
      tma_prefetch_desc(&zmap);
      int it = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
        const int s = it % kOutBufs;
        for (int d = (it == 0 ? 1 : max(tl.pf, 1)); d <= tl.pf; ++d) {
          const int tp = t + d * static_cast<int>(gridDim.x);
          if (tp < ntiles) {
            int pb, pu, pv;
            tl.tile(tp, pb, pu, pv);
            tma_prefetch_l2_4d(&zmap, 0, pv, pu, pb);
            tma_prefetch_l2_4d(&zmap, 64, pv, pu, pb);
          }
        }
        if (!mbar_wait(&z_empty[s], ((it / kOutBufs) & 1) ^ 1, err,
                       err_code(KERNEL_OUTPUT, ROLE_PRODUCER, 2)))
          break;
        int b, u0, v0;
        tl.tile(t, b, u0, v0);
        uint8_t* zs = sSlots + s * kSlot;
        mbar_arrive_expect_tx(&full_z[s], kZTile);
        tma_load_4d(&zmap, &full_z[s], zs, 0, v0, u0, b);
        tma_load_4d(&zmap, &full_z[s], zs + kHalfTile, 64, v0, u0, b);
      }
      for (int i = (it > kOutBufs ? it - kOutBufs : 0); i < it; ++i)
        mbar_wait_drain(&full_z[i % kOutBufs], (i / kOutBufs) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_z = idesc_f16(0, 128, 128, 0, 0);
      constexpr uint32_t idesc_x = idesc_f16(0, 128, 128, 1, 0);  // A (x) is MN-major
      const uint32_t wbase = smem_u32(sW);
      bool ok = mbar_wait(w_full, 0, err, err_code(KERNEL_OUTPUT, ROLE_MMA, 1));
      tc_fence_after();
      int it = 0;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x, ++it) {
        const int s = it % kOutBufs;
        const uint32_t ph = (it / kOutBufs) & 1;
        if (!mbar_wait(&a_ready[s], ph, err, err_code(KERNEL_OUTPUT, ROLE_MMA, 2)) ||
            !mbar_wait(&tmem_empty[s], ph ^ 1, err, err_code(KERNEL_OUTPUT, ROLE_MMA, 3))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t zs = smem_u32(sSlots + s * kSlot);
        const uint32_t xs = zs + kZTile;
        const uint32_t d = tmem_base + s * 256;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // gate projection: z (K-major) x W_g'
          const uint64_t ad = kmajor_desc(zs + (kk >> 2) * kHalfTile + (kk & 3) * 32);
          const uint64_t bd = kmajor_desc(wbase + (kk >> 2) * 32768 + (kk & 3) * 32);
          umma_f16(d, ad, bd, idesc_z, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // output projection: x (MN-major) x W_o'
          const uint64_t ad = sw128_desc(xs + kk * 2048, kHalfTile, 1024);
          const uint64_t bd = kmajor_desc(wbase + (kk >> 2) * 32768 + 16384 + (kk & 3) * 32);
          umma_f16(d + 128, ad, bd, idesc_x, kk > 0 ? 1u : 0u);
        }
        umma_commit(&tmem_full[s]);
        umma_commit(&x_empty[s]);
      }
      umma_commit(mma_drain);
      mbar_wait_drain(mma_drain, 0);
    }
  } else if (warp < 6) {
    const int row = threadIdx.x - 64;
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const int s = it % kOutBufs;
      int b, u0, v0;
      tl.tile(t, b, u0, v0);
      const int u = u0 + row / tl.vt, v = v0 + row % tl.vt;
      const bool valid = (u < tl.R) && (v < tl.S);
      // mask and the z LayerNorm statistics written by the input stage, loaded before
      // the wait so their latency hides behind the TMA
      const size_t zi = (static_cast<size_t>(b) * tl.R + u) * tl.S + v;
      float m = 0.f;
      float2 zst = make_float2(0.f, 0.f);
      if (valid) {
        m = mask ? __ldg(mask + zi) : 1.f;
        zst = __ldg(zstats + zi);
      }
      // warp-uniform: the statistics below exchange partial sums between lanes
      if (!mbar_wait_warp(&full_x[s], (it / kOutBufs) & 1, err, err_code(KERNEL_OUTPUT, ROLE_TRANSFORM, 1)))
        break;
      uint8_t* zs = sSlots + s * kSlot;
      const uint8_t* xs = zs + kZTile;
      const float inv_c = 1.0f / kC;
      float dm;
      // x column statistics of the MN-major x tile, two positions per thread pair:
      // threads row and row ^ 1 own positions pr, pr + 1 and split the channels in
      // halves; each reads half2 words (both positions of one channel), accumulates the
      // two positions in the lanes of FADD2 / FFMA2, and the halves are then combined
      // with the partner by shuffle. Channel 0 of each position is its shift.
      const int pr = row & ~1, chh = row & 1;
      const int h = pr >> 6, e = pr & 63;
      const uint8_t* xcol = xs + h * kHalfTile + (e & 7) * 2;
      const float2 shift = __half22float2(*reinterpret_cast<const __half2*>(xcol + sw128_off(0, e >> 3)));
      const float2 nshift = make_float2(-shift.x, -shift.y);
      float2 a1[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      float2 a2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll 8
      for (int c = chh * (kC / 2); c < chh * (kC / 2) + kC / 2; c += 2) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const float2 xv = __half22float2(*reinterpret_cast<const __half2*>(xcol + sw128_off(c + k, e >> 3)));
          const float2 d = __fadd2_rn(xv, nshift);
          a1[k] = __fadd2_rn(a1[k], d);
          a2[k] = __ffma2_rn(d, d, a2[k]);
        }
      }
      float2 s1 = __fadd2_rn(a1[0], a1[1]), s2 = __fadd2_rn(a2[0], a2[1]);
      s1.x += __shfl_xor_sync(0xffffffffu, s1.x, 1);
      s1.y += __shfl_xor_sync(0xffffffffu, s1.y, 1);
      s2.x += __shfl_xor_sync(0xffffffffu, s2.x, 1);
      s2.y += __shfl_xor_sync(0xffffffffu, s2.y, 1);
      dm = (chh ? s1.y : s1.x) * inv_c;
      const float mean_x = (chh ? shift.y : shift.x) + dm;
      const float var_x = fmaxf((chh ? s2.y : s2.x) * inv_c - dm * dm, 0.f);
      if (!mbar_wait(&full_z[s], (it / kOutBufs) & 1, err, err_code(KERNEL_OUTPUT, ROLE_TRANSFORM, 2)))
        break;
      if (z_bf16) {   // bf16 -> fp16 in place (exact inside fp16 range): the MMA operand
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          uint4* p = reinterpret_cast<uint4*>(zs + (q >> 3) * kHalfTile + sw128_off(row, q & 7));
          float f[8];
          unpack8(*p, 1, f);
          *p = make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]), pack_half2(f[4], f[5]),
                          pack_half2(f[6], f[7]));
        }
      }
      const float sa = zst.y, mean_z = zst.x;   // sa = m * rstd of z*m (input stage)
      const float rx = rsqrtf(var_x + eps_out);
      // gate pre-activation halves: g/2 = (sa/2) acc_g + (-sa mean) (u_g/2) + v_g/2
      sStats[(it % kStatRing) * 128 + row] = make_float4(0.5f * sa, -sa * mean_z, rx, -rx * mean_x);
      sMask[(it % kStatRing) * 128 + row] = m;
      fence_proxy_async_smem();
      mbar_arrive(&a_ready[s]);
    }
  } else {
    const int sub = warp & 3;
    const int nhalf = (warp - 6) >> 2;   // output channels [64 * nhalf, 64 * nhalf + 64)
    const int row = sub * 32 + lane;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(sub * 32) << 16);
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const int s = it % kOutBufs;
      const uint32_t ph = (it / kOutBufs) & 1;
      if (!mbar_wait_warp(&a_ready[s], ph, err, err_code(KERNEL_OUTPUT, ROLE_EPILOGUE, 1)) ||
          !mbar_wait_warp(&tmem_full[s], ph, err, err_code(KERNEL_OUTPUT, ROLE_EPILOGUE, 2)))
        break;
      tc_fence_after();
      int b, u0, v0;
      tl.tile(t, b, u0, v0);
      const int u = u0 + row / tl.vt, v = v0 + row % tl.vt;
      const bool valid = (u < tl.R) && (v < tl.S);
      const size_t elem0 = ((static_cast<size_t>(b) * tl.R + u) * tl.S + v) * kC;
      const float4 st = sStats[(it % kStatRing) * 128 + row];
      const float m = sMask[(it % kStatRing) * 128 + row];
      const float hm = 0.5f * m, m2 = m * m;
      const float2 hm2 = make_float2(hm, hm), m22 = make_float2(m2, m2);
      const float2 stx2 = make_float2(st.x, st.x), sty2 = make_float2(st.y, st.y);
      const float2 stz2 = make_float2(st.z, st.z), stw2 = make_float2(st.w, st.w);
      uint8_t* zs = sSlots + s * kSlot;
      // four 16-column sub-chunks per warp; the TMEM load of sub-chunk k+1 is in
      // flight while sub-chunk k is computed
      uint32_t gr[2][16], orr[2][16];
      tmem_ld16_nowait(lane_base + s * 256 + nhalf * 64, gr[0]);
      tmem_ld16_nowait(lane_base + s * 256 + 128 + nhalf * 64, orr[0]);
      tmem_wait_ld();
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int cur = k & 1;
        const int n0 = nhalf * 64 + k * 16;    // first output channel of this sub-chunk
        if (k < 3) {
          tmem_ld16_nowait(lane_base + s * 256 + n0 + 16, gr[cur ^ 1]);
          tmem_ld16_nowait(lane_base + s * 256 + 128 + n0 + 16, orr[cur ^ 1]);
        }
        float zv[16];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int chunk = (n0 >> 3) + q;  // 16-byte chunk of the 256-byte z row
          float f[8];
          unpack8(*reinterpret_cast<const uint4*>(zs + (chunk >> 3) * kHalfTile +
                                                  sw128_off(row, chunk & 7)), 0, f);
#pragma unroll
          for (int e2 = 0; e2 < 8; ++e2) zv[q * 8 + e2] = f[e2];
        }
        float r[16];
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          // out = m^2 z (residual) + m * o * sigmoid(g), sigmoid(g) = (1 + tanh(g/2)) / 2,
          // two channels per packed fp32x2 operation
          const float4 cg = sUV[n0 + i], co = sUV[n0 + i + 1];
          const float2 to = __ffma2_rn(stz2, make_float2(__uint_as_float(orr[cur][i]), __uint_as_float(orr[cur][i + 1])),
                                       __ffma2_rn(stw2, make_float2(co.x, co.y), make_float2(co.z, co.w)));
          const float2 hmo = __fmul2_rn(hm2, to);
          const float2 tg = __ffma2_rn(stx2, make_float2(__uint_as_float(gr[cur][i]), __uint_as_float(gr[cur][i + 1])),
                                       __ffma2_rn(sty2, make_float2(cg.x, cg.y), make_float2(cg.z, cg.w)));
          const float2 th = make_float2(tanh_mufu(tg.x), tanh_mufu(tg.y));
          const float2 base = residual ? __ffma2_rn(m22, make_float2(zv[i], zv[i + 1]), hmo) : hmo;
          const float2 rr = __ffma2_rn(hmo, th, base);
          r[i] = rr.x;
          r[i + 1] = rr.y;
        }
        if (OUT_DT == 0) {
          if (valid) {
            float4* po = reinterpret_cast<float4*>(static_cast<float*>(out) + elem0 + n0);
#pragma unroll
            for (int q = 0; q < 4; ++q) po[q] = make_float4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
          }
        } else {
          // 16-bit output: overwrite the z chunks just read (same thread, same
          // addresses) so the slot holds the out tile in the z tile's layout
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int chunk = (n0 >> 3) + q;
            uint4 o;
            uint32_t* w = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
            for (int e2 = 0; e2 < 4; ++e2)
              w[e2] = OUT_DT == 1 ? pack_half2(r[q * 8 + 2 * e2], r[q * 8 + 2 * e2 + 1])
                                  : pack_bf162(r[q * 8 + 2 * e2], r[q * 8 + 2 * e2 + 1]);
            *reinterpret_cast<uint4*>(zs + (chunk >> 3) * kHalfTile + sw128_off(row, chunk & 7)) = o;
          }
        }
        if (k < 3) tmem_wait_ld();
      }
      tc_fence_before();
      if (OUT_DT != 0) {
        // TMA-store this warp's 32 rows x 64 channels (clipped at the tensor edges)
        fence_proxy_async_smem();
        __syncwarp();
        const int r0 = sub * 32;
        const int uw = u0 + r0 / tl.vt, vw = v0 + r0 % tl.vt;
        if (lane == 0) {
          if (uw < tl.R && vw < tl.S) {
            tma_store_4d(&omap, zs + nhalf * kHalfTile + r0 * 128, nhalf * 64, vw, uw, b);
            bulk_commit();
          }
          bulk_wait_read0();   // slot may be refilled once the store has read it
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&tmem_empty[s]);
        mbar_arrive(&z_empty[s]);
      }
    }
  }

  if (OUT_DT != 0 && warp >= 6 && (threadIdx.x & 31) == 0) bulk_wait0();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace

size_t output_stage_smem_bytes() { return kSmemBytes; }

cudaError_t launch_output_stage(const CUtensorMap& zmap, const CUtensorMap& xmap,
                                const CUtensorMap& wmap, const CUtensorMap& omap, const float* mask,
                                const float2* zstats, const float* u_g,
                                const float* v_g, const float* u_o, const float* v_o, void* out,
                                int out_dtype, const PosTiling& tl, int residual, int z_bf16,
                                float eps_in, float eps_out, int* err, int grid,
                                cudaStream_t stream) {
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t e =
        set_smem_once(reinterpret_cast<const void*>(kern), kSmemBytes);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, dim3(grid), dim3(kOutThreads), kSmemBytes, stream, nullptr, 0, zmap, xmap,
                      wmap, omap, mask, zstats, u_g, v_g, u_o, v_o, out, tl, residual, z_bf16,
                      eps_in, eps_out, err);
  };
  switch (out_dtype) {
    case 0: return go(output_stage_kernel<0>);
    case 1: return go(output_stage_kernel<1>);
    case 2: return go(output_stage_kernel<2>);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ftm
