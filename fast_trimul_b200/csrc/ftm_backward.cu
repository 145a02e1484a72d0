// Per-position kernels of the training backward (c_z = c_h = 128).
//
// The backward of the reference's training path (fast_trimul/_kernels.py:468-488, the
// autograd of `_torch_forward`, :532-547) splits into
//   * per-position GEMMs (projections and their transposes): cuBLAS through torch;
//   * the two N^3 products of the contraction: the tcgen05 contraction kernel;
//   * everything elementwise / per-row: these kernels, each one pass over HBM, fusing
//     what autograd runs as a chain of elementwise kernels and strided layout copies.
// Layouts: positions p = (b * N + u) * N + v in position-major rows of 128 channels;
// planes [b][c][u][v] (the contraction's channel-major layout). Plane <-> position tiles
// are transposed through shared memory (32 positions x 128 channels per tile).
//
// Gradients are computed from a pre-scaled output gradient (the caller divides it by its
// largest magnitude and multiplies every result back), so the fp16 intermediates keep
// their precision whatever the loss scale.
#include "ftm_kernels.h"

namespace ftm {
namespace {

constexpr int kTile = 32;              // positions per plane tile
constexpr int kH = 640;                // columns of H / dPGZ: [p_a g_a p_b g_b | g_z]

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void load4(const void* base, int dtype, size_t idx, float (&f)[4]) {
  if (dtype == FTM_F32) {
    const float4 v = *reinterpret_cast<const float4*>(static_cast<const float*>(base) + idx);
    f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
  } else {
    const uint2 v = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(base) + idx);
    const uint32_t w[2] = {v.x, v.y};
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      float2 t;
      if (dtype == FTM_F16) t = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
      else t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
      f[2 * k] = t.x;
      f[2 * k + 1] = t.y;
    }
  }
}

__device__ __forceinline__ void store4(void* base, int dtype, size_t idx, const float (&f)[4]) {
  if (dtype == FTM_F32) {
    *reinterpret_cast<float4*>(static_cast<float*>(base) + idx) = make_float4(f[0], f[1], f[2], f[3]);
  } else if (dtype == FTM_F16) {
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(base) + idx) =
        make_uint2(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]));
  } else {
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(base) + idx) =
        make_uint2(pack_bf162(f[0], f[1]), pack_bf162(f[2], f[3]));
  }
}

__device__ __forceinline__ float sigmoidf(float x) { return 1.0f / (1.0f + __expf(-x)); }

// ---------------------------------------------------------------- input LayerNorm
// zn = LayerNorm(z * m) as fp16 rows, stats = (mean, rstd) of z * m. One warp per
// position, four channels per lane.
__global__ void ln_in_kernel(const void* __restrict__ z, int z_dtype, const float* __restrict__ mask,
                             const float* __restrict__ gamma, const float* __restrict__ beta,
                             float eps, __half* __restrict__ zn, float2* __restrict__ stats,
                             long long P) {
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const float4 g4 = *reinterpret_cast<const float4*>(gamma + 4 * lane);
  const float4 b4 = *reinterpret_cast<const float4*>(beta + 4 * lane);
  for (long long p = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; p < P;
       p += warps) {
    float f[4];
    load4(z, z_dtype, static_cast<size_t>(p) * kC + 4 * lane, f);
    const float m = mask ? mask[p] : 1.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) f[k] *= m;
    const float mean = warp_sum(f[0] + f[1] + f[2] + f[3]) * (1.f / kC);
    float sq = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) sq += (f[k] - mean) * (f[k] - mean);
    const float rstd = rsqrtf(warp_sum(sq) * (1.f / kC) + eps);
    float o[4] = {(f[0] - mean) * rstd * g4.x + b4.x, (f[1] - mean) * rstd * g4.y + b4.y,
                  (f[2] - mean) * rstd * g4.z + b4.z, (f[3] - mean) * rstd * g4.w + b4.w};
    store4(zn, FTM_F16, static_cast<size_t>(p) * kC + 4 * lane, o);
    if (lane == 0) stats[p] = make_float2(mean, rstd);
  }
}

// Plane tile (b, u, v0 .. v0 + 31) x 128 channels of an fp16 plane -> shared memory
// tile[c][j], 8 positions (16 bytes) per load where the row allows it.
__device__ __forceinline__ void load_plane_tile(const __half* __restrict__ plane, int b, int u,
                                                int v0, int N, float (*tile)[kTile + 1]) {
  const bool vec = (v0 + kTile <= N) && (N % 8 == 0);
  if (vec) {
    for (int idx = threadIdx.x; idx < kC * (kTile / 8); idx += blockDim.x) {
      const int c = idx / (kTile / 8), j8 = (idx % (kTile / 8)) * 8;
      const uint4 w = *reinterpret_cast<const uint4*>(
          plane + ((static_cast<size_t>(b) * kC + c) * N + u) * N + v0 + j8);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ws[q]));
        tile[c][j8 + 2 * q] = f.x;
        tile[c][j8 + 2 * q + 1] = f.y;
      }
    }
    return;
  }
  for (int idx = threadIdx.x; idx < kC * kTile; idx += blockDim.x) {
    const int c = idx / kTile, j = idx % kTile, v = v0 + j;
    tile[c][j] = v < N ? __half2float(plane[((static_cast<size_t>(b) * kC + c) * N + u) * N + v]) : 0.f;
  }
}

// Block-wide sums of per-thread channel partials (four channels per lane, `groups` groups
// of 128 channels) written as one row of `partial`.
template <int G>
__device__ __forceinline__ void write_partials(float (*red)[G * kC], const float (&acc)[G][4],
                                               float* partial) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int k = 0; k < 4; ++k) red[warp][g * kC + 4 * lane + k] = acc[g][k];
  __syncthreads();
  for (int c = threadIdx.x; c < G * kC; c += blockDim.x) {
    float s = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += red[w][c];
    partial[static_cast<size_t>(blockIdx.x) * G * kC + c] = s;
  }
}

// ---------------------------------------------------------------- output LayerNorm
// xn = LayerNorm(x) rows (fp16) and stats (mean, rstd) from the channel-major x plane.
__global__ void x_ln_kernel(const __half* __restrict__ xplane, const float* __restrict__ gamma,
                            const float* __restrict__ beta, float eps, __half* __restrict__ xn,
                            float2* __restrict__ stats, int B, int N) {
  __shared__ float tile[kC][kTile + 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int vt = (N + kTile - 1) / kTile;
  const long long tiles = static_cast<long long>(B) * N * vt;
  const float4 g4 = *reinterpret_cast<const float4*>(gamma + 4 * lane);
  const float4 b4 = *reinterpret_cast<const float4*>(beta + 4 * lane);
  for (long long t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int b = static_cast<int>(t / (static_cast<long long>(N) * vt));
    const int rem = static_cast<int>(t % (static_cast<long long>(N) * vt));
    const int u = rem / vt, v0 = (rem % vt) * kTile;
    __syncthreads();
    load_plane_tile(xplane, b, u, v0, N, tile);
    __syncthreads();
    for (int j = warp; j < kTile; j += blockDim.x >> 5) {
      const int v = v0 + j;
      if (v >= N) continue;
      const size_t p = (static_cast<size_t>(b) * N + u) * N + v;
      float f[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) f[k] = tile[4 * lane + k][j];
      const float mean = warp_sum(f[0] + f[1] + f[2] + f[3]) * (1.f / kC);
      float sq = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) sq += (f[k] - mean) * (f[k] - mean);
      const float rstd = rsqrtf(warp_sum(sq) * (1.f / kC) + eps);
      float o[4] = {(f[0] - mean) * rstd * g4.x + b4.x, (f[1] - mean) * rstd * g4.y + b4.y,
                    (f[2] - mean) * rstd * g4.z + b4.z, (f[3] - mean) * rstd * g4.w + b4.w};
      store4(xn, FTM_F16, p * kC + 4 * lane, o);
      if (lane == 0) stats[p] = make_float2(mean, rstd);
    }
  }
}

// ---------------------------------------------------------------- output gate
// out = (zm + delta) * m, delta = sigmoid(gz) * o. With dd = dout * m:
//   do = dd * sigmoid(gz),  dgz = dd * o * sigmoid(gz) * (1 - sigmoid(gz)).
// O, H hold the GEMM results without biases.
__global__ void gate_bwd_kernel(const __half* __restrict__ O, const float* __restrict__ b_o,
                                const __half* __restrict__ H, const float* __restrict__ b_g,
                                const void* __restrict__ gout, int g_dtype,
                                const float* __restrict__ g_scale_p,
                                const float* __restrict__ mask, __half* __restrict__ dO,
                                __half* __restrict__ dPGZ, float* __restrict__ partial, long long P) {
  __shared__ float red[8][2 * kC];
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const float4 bo = *reinterpret_cast<const float4*>(b_o + 4 * lane);
  const float4 bg = *reinterpret_cast<const float4*>(b_g + 4 * lane);
  const float bo_[4] = {bo.x, bo.y, bo.z, bo.w}, bg_[4] = {bg.x, bg.y, bg.z, bg.w};
  for (long long p = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; p < P;
       p += warps) {
    float o[4], gz[4], g[4];
    load4(O, FTM_F16, static_cast<size_t>(p) * kC + 4 * lane, o);
    load4(H, FTM_F16, static_cast<size_t>(p) * kH + 512 + 4 * lane, gz);
    load4(gout, g_dtype, static_cast<size_t>(p) * kC + 4 * lane, g);
    const float m = (mask ? mask[p] : 1.f) * *g_scale_p;
    float dov[4], dgz[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float s = sigmoidf(gz[k] + bg_[k]);
      const float dd = g[k] * m;
      dov[k] = dd * s;
      dgz[k] = dd * (o[k] + bo_[k]) * s * (1.f - s);
      acc[0][k] += dov[k];
      acc[1][k] += dgz[k];
    }
    store4(dO, FTM_F16, static_cast<size_t>(p) * kC + 4 * lane, dov);
    store4(dPGZ, FTM_F16, static_cast<size_t>(p) * kH + 512 + 4 * lane, dgz);
  }
  write_partials<2>(red, acc, partial);
}

// ---------------------------------------------------------------- output LayerNorm backward
// dx = rstd * (gy - mean(gy) - xh * mean(gy * xh)), gy = dxn * gamma, written to the
// channel-major fp32 plane; per-block partial sums of dxn * xh (dgamma) and dxn (dbeta).
__global__ void x_ln_bwd_kernel(const __half* __restrict__ xplane, const float2* __restrict__ stats,
                                const __half* __restrict__ dxn, const float* __restrict__ gamma,
                                float* __restrict__ dxplane, float* __restrict__ partial, int B,
                                int N) {
  __shared__ float tile[kC][kTile + 1];
  __shared__ float red[8][2 * kC];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int vt = (N + kTile - 1) / kTile;
  const long long tiles = static_cast<long long>(B) * N * vt;
  const float4 g4 = *reinterpret_cast<const float4*>(gamma + 4 * lane);
  const float gm[4] = {g4.x, g4.y, g4.z, g4.w};
  float dg[4] = {0.f, 0.f, 0.f, 0.f}, db[4] = {0.f, 0.f, 0.f, 0.f};
  for (long long t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int b = static_cast<int>(t / (static_cast<long long>(N) * vt));
    const int rem = static_cast<int>(t % (static_cast<long long>(N) * vt));
    const int u = rem / vt, v0 = (rem % vt) * kTile;
    __syncthreads();
    load_plane_tile(xplane, b, u, v0, N, tile);
    __syncthreads();
    for (int j = warp; j < kTile; j += blockDim.x >> 5) {
      const int v = v0 + j;
      if (v >= N) continue;
      const size_t p = (static_cast<size_t>(b) * N + u) * N + v;
      const float2 st = stats[p];
      float dy[4], xh[4], gy[4];
      load4(dxn, FTM_F16, p * kC + 4 * lane, dy);
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        xh[k] = (tile[4 * lane + k][j] - st.x) * st.y;
        gy[k] = dy[k] * gm[k];
        s1 += gy[k];
        s2 += gy[k] * xh[k];
        dg[k] += dy[k] * xh[k];
        db[k] += dy[k];
      }
      s1 = warp_sum(s1) * (1.f / kC);
      s2 = warp_sum(s2) * (1.f / kC);
#pragma unroll
      for (int k = 0; k < 4; ++k) tile[4 * lane + k][j] = st.y * (gy[k] - s1 - xh[k] * s2);
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < kC * kTile; idx += blockDim.x) {
      const int c = idx / kTile, j = idx % kTile, v = v0 + j;
      if (v < N) dxplane[((static_cast<size_t>(b) * kC + c) * N + u) * N + v] = tile[c][j];
    }
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    red[warp][4 * lane + k] = dg[k];
    red[warp][kC + 4 * lane + k] = db[k];
  }
  __syncthreads();
  for (int c = threadIdx.x; c < 2 * kC; c += blockDim.x) {
    float s = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += red[w][c];
    partial[static_cast<size_t>(blockIdx.x) * 2 * kC + c] = s;
  }
}

// ---------------------------------------------------------------- input gates backward
// a = p_a sigmoid(g_a) (same for b): dp = da sigmoid(g), dg = da p sigmoid(g)(1 - sigmoid(g)).
// da, db come as fp16 planes in position order [b][c][u][v], scaled by `dscale`.
__global__ void gates_in_bwd_kernel(const __half* __restrict__ dA, const __half* __restrict__ dB,
                                    const float* __restrict__ dscale_p, const __half* __restrict__ H,
                                    const float* __restrict__ b_in, __half* __restrict__ dPGZ,
                                    float* __restrict__ partial, int B, int N) {
  __shared__ float ta[kC][kTile + 1];
  __shared__ float tb[kC][kTile + 1];
  float acc[4][4] = {};
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int vt = (N + kTile - 1) / kTile;
  const long long tiles = static_cast<long long>(B) * N * vt;
  float bias[4][4];
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int k = 0; k < 4; ++k) bias[q][k] = b_in[q * kC + 4 * lane + k];
  for (long long t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int b = static_cast<int>(t / (static_cast<long long>(N) * vt));
    const int rem = static_cast<int>(t % (static_cast<long long>(N) * vt));
    const int u = rem / vt, v0 = (rem % vt) * kTile;
    __syncthreads();
    load_plane_tile(dA, b, u, v0, N, ta);
    load_plane_tile(dB, b, u, v0, N, tb);
    __syncthreads();
    for (int j = warp; j < kTile; j += blockDim.x >> 5) {
      const int v = v0 + j;
      if (v >= N) continue;
      const size_t p = (static_cast<size_t>(b) * N + u) * N + v;
#pragma unroll
      for (int half = 0; half < 2; ++half) {   // a then b
        float pr[4], gr[4], dpv[4], dgv[4];
        load4(H, FTM_F16, p * kH + half * 256 + 4 * lane, pr);
        load4(H, FTM_F16, p * kH + half * 256 + 128 + 4 * lane, gr);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float d = (half ? tb : ta)[4 * lane + k][j] * *dscale_p;
          const float pv = pr[k] + bias[2 * half][k];
          const float s = sigmoidf(gr[k] + bias[2 * half + 1][k]);
          dpv[k] = d * s;
          dgv[k] = d * pv * s * (1.f - s);
          acc[2 * half][k] += dpv[k];
          acc[2 * half + 1][k] += dgv[k];
        }
        store4(dPGZ, FTM_F16, p * kH + half * 256 + 4 * lane, dpv);
        store4(dPGZ, FTM_F16, p * kH + half * 256 + 128 + 4 * lane, dgv);
      }
    }
  }
  __syncthreads();
  // the tiles are free now: reuse them as the reduction buffer (8 warps x 512 floats)
  write_partials<4>(reinterpret_cast<float (*)[4 * kC]>(&ta[0][0]), acc, partial);
}

// ---------------------------------------------------------------- input LayerNorm backward
// zm = z * m, zn = LN(zm); out = (zm + delta) * m (residual) or delta * m:
//   dzm = rstd (gy - mean(gy) - xh mean(gy xh)) [+ dout * m],  dz = dzm * m,
// gy = dzn * gamma. Per-block partial sums of dzn * xh and dzn.
__global__ void ln_in_bwd_kernel(const void* __restrict__ z, int z_dtype,
                                 const float* __restrict__ mask, const float2* __restrict__ stats,
                                 const __half* __restrict__ dzn, const float* __restrict__ gamma,
                                 const void* __restrict__ gout, int g_dtype,
                                 const float* __restrict__ g_scale_p, int residual, void* __restrict__ dz, int dz_dtype,
                                 float* __restrict__ partial, long long P) {
  __shared__ float red[8][2 * kC];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const float4 g4 = *reinterpret_cast<const float4*>(gamma + 4 * lane);
  const float gm[4] = {g4.x, g4.y, g4.z, g4.w};
  float dg[4] = {0.f, 0.f, 0.f, 0.f}, db[4] = {0.f, 0.f, 0.f, 0.f};
  for (long long p = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; p < P;
       p += warps) {
    const float m = mask ? mask[p] : 1.f;
    const float2 st = stats[p];
    float zf[4], dy[4], xh[4], gy[4];
    load4(z, z_dtype, static_cast<size_t>(p) * kC + 4 * lane, zf);
    load4(dzn, FTM_F16, static_cast<size_t>(p) * kC + 4 * lane, dy);
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      xh[k] = (zf[k] * m - st.x) * st.y;
      gy[k] = dy[k] * gm[k];
      s1 += gy[k];
      s2 += gy[k] * xh[k];
      dg[k] += dy[k] * xh[k];
      db[k] += dy[k];
    }
    s1 = warp_sum(s1) * (1.f / kC);
    s2 = warp_sum(s2) * (1.f / kC);
    float res[4] = {0.f, 0.f, 0.f, 0.f};
    if (residual) load4(gout, g_dtype, static_cast<size_t>(p) * kC + 4 * lane, res);
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = (st.y * (gy[k] - s1 - xh[k] * s2) + res[k] * m * *g_scale_p) * m;
    store4(dz, dz_dtype, static_cast<size_t>(p) * kC + 4 * lane, o);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    red[warp][4 * lane + k] = dg[k];
    red[warp][kC + 4 * lane + k] = db[k];
  }
  __syncthreads();
  for (int c = threadIdx.x; c < 2 * kC; c += blockDim.x) {
    float s = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += red[w][c];
    partial[static_cast<size_t>(blockIdx.x) * 2 * kC + c] = s;
  }
}

int launched(cudaError_t e) { return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? FTM_OK : FTM_LAUNCH_FAILED; }

bool dtype_ok(int d) { return d == FTM_F32 || d == FTM_F16 || d == FTM_BF16; }

}  // namespace

// Grid of the per-position kernels: a fixed number of 256-thread blocks per SM, so the
// per-block partial sums stay few (partial buffers: ftm_bwd_partial_blocks() x 256 floats).
int bwd_blocks() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms * 4;
}

}  // namespace ftm

using namespace ftm;

extern "C" {

int ftm_bwd_partial_blocks(void) { return bwd_blocks(); }

int ftm_bwd_ln_in(const void* z, int32_t z_dtype, const float* mask, const float* gamma,
                  const float* beta, float eps, void* zn, float* stats, int64_t positions,
                  ftm_stream_t stream) {
  if (!z || !gamma || !beta || !zn || !stats || positions < 1 || !dtype_ok(z_dtype))
    return FTM_BAD_ARGUMENT;
  ln_in_kernel<<<bwd_blocks(), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      z, z_dtype, mask, gamma, beta, eps, static_cast<__half*>(zn), reinterpret_cast<float2*>(stats),
      positions);
  return launched(cudaSuccess);
}

int ftm_bwd_x_ln(const void* xplane, const float* gamma, const float* beta, float eps, void* xn,
                 float* stats, int32_t batch, int32_t n, ftm_stream_t stream) {
  if (!xplane || !gamma || !beta || !xn || !stats || batch < 1 || n < 1) return FTM_BAD_ARGUMENT;
  x_ln_kernel<<<bwd_blocks(), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(xplane), gamma, beta, eps, static_cast<__half*>(xn),
      reinterpret_cast<float2*>(stats), batch, n);
  return launched(cudaSuccess);
}

int ftm_bwd_gate(const void* O, const float* b_o, const void* H, const float* b_g, const void* gout,
                 int32_t g_dtype, const float* g_scale, const float* mask, void* dO, void* dPGZ,
                 float* partial, int64_t positions, ftm_stream_t stream) {
  if (!O || !b_o || !H || !b_g || !gout || !g_scale || !dO || !dPGZ || !partial || positions < 1 ||
      !dtype_ok(g_dtype))
    return FTM_BAD_ARGUMENT;
  gate_bwd_kernel<<<bwd_blocks(), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(O), b_o, static_cast<const __half*>(H), b_g, gout, g_dtype, g_scale,
      mask, static_cast<__half*>(dO), static_cast<__half*>(dPGZ), partial, positions);
  return launched(cudaSuccess);
}

int ftm_bwd_x_ln_bwd(const void* xplane, const float* stats, const void* dxn, const float* gamma,
                     float* dxplane, float* partial, int32_t batch, int32_t n, ftm_stream_t stream) {
  if (!xplane || !stats || !dxn || !gamma || !dxplane || !partial || batch < 1 || n < 1)
    return FTM_BAD_ARGUMENT;
  x_ln_bwd_kernel<<<bwd_blocks(), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(xplane), reinterpret_cast<const float2*>(stats),
      static_cast<const __half*>(dxn), gamma, dxplane, partial, batch, n);
  return launched(cudaSuccess);
}

int ftm_bwd_gates_in(const void* dA, const void* dB, const float* dscale, const void* H, const float* b_in,
                     void* dPGZ, float* partial, int32_t batch, int32_t n, ftm_stream_t stream) {
  if (!dA || !dB || !dscale || !H || !b_in || !dPGZ || !partial || batch < 1 || n < 1) return FTM_BAD_ARGUMENT;
  gates_in_bwd_kernel<<<bwd_blocks(), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(dA), static_cast<const __half*>(dB), dscale,
      static_cast<const __half*>(H), b_in, static_cast<__half*>(dPGZ), partial, batch, n);
  return launched(cudaSuccess);
}

int ftm_bwd_ln_in_bwd(const void* z, int32_t z_dtype, const float* mask, const float* stats,
                      const void* dzn, const float* gamma, const void* gout, int32_t g_dtype,
                      const float* g_scale, int32_t residual, void* dz, int32_t dz_dtype, float* partial,
                      int64_t positions, ftm_stream_t stream) {
  if (!z || !stats || !dzn || !gamma || !gout || !g_scale || !dz || !partial || positions < 1 ||
      !dtype_ok(z_dtype) || !dtype_ok(g_dtype) || !dtype_ok(dz_dtype))
    return FTM_BAD_ARGUMENT;
  ln_in_bwd_kernel<<<bwd_blocks(), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      z, z_dtype, mask, reinterpret_cast<const float2*>(stats), static_cast<const __half*>(dzn),
      gamma, gout, g_dtype, g_scale, residual, dz, dz_dtype, partial, positions);
  return launched(cudaSuccess);
}

}  // extern "C"
