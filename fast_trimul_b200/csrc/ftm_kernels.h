// Internal launch interface between the C ABI (ftm_api.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ftm_common.cuh"
#include "../../include/fast_trimul_b200.h"

namespace ftm {

// Launch with programmatic stream serialisation (FTM_PDL=0 turns it off): the kernel's
// set-up overlaps the tail of the previous kernel on the stream; the kernels call
// grid_dep_wait() before their first global access.
bool pdl_enabled();
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per kernel and device
cudaError_t set_smem_once(const void* kern, int bytes);
template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       const cudaLaunchAttribute* extra, int n_extra, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[4];
  int n = 0;
  for (int i = 0; i < n_extra && n < 3; ++i) attr[n++] = extra[i];
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  return e != cudaSuccess ? e : cudaGetLastError();
}

// Packed parameter buffer (built by ftm_pack_params), byte offsets for C = c_z = c_h.
struct PackedLayout {
  size_t w_in, w_out, u_in, v_in, u_g, v_g, u_o, v_o, total;
  static PackedLayout make(int c_z, int c_h) {
    auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
    PackedLayout L{};
    size_t off = 0;
    L.w_in = off;  off = up(off + size_t(4) * c_h * c_z * 2);            // [a_p;a_g;b_p;b_g] x c_z, fp16
    L.w_out = off; off = up(off + size_t(c_z) * c_z * 2 + size_t(c_z) * c_h * 2);  // [W_g'; W_o'] fp16
    L.u_in = off;  off = up(off + size_t(4) * c_h * 4);
    L.v_in = off;  off = up(off + size_t(4) * c_h * 4);
    L.u_g = off;   off = up(off + size_t(c_z) * 4);
    L.v_g = off;   off = up(off + size_t(c_z) * 4);
    L.u_o = off;   off = up(off + size_t(c_z) * 4);
    L.v_o = off;   off = up(off + size_t(c_z) * 4);
    L.total = off;
    return L;
  }
};

constexpr int kC = 128;            // c_z == c_h supported by the tensor-core kernels
constexpr int kInThreads = 576;    // producer, MMA, 8 transform, 8 epilogue warps
constexpr int kInBufs = 2;
constexpr int kOutThreads = 448;   // producer, MMA, 4 transform, 8 epilogue warps
constexpr int kOutBufs = 2;
constexpr int kCtThreads = 192;    // producer, MMA, 4 epilogue warps
constexpr int kCtStages = 4;
constexpr int kCtBM = 128, kCtBN = 256, kCtBK = 64;

size_t input_stage_smem_bytes();
size_t output_stage_smem_bytes();
size_t contraction_smem_bytes();

// Destinations of the input stage's a / b stores: one tensor map per destination
// rank (one map, the local planes, when not sharded). Channel c of a tile goes to map
// c / lq at channel coordinate c % lq and outer coordinate blk_base + batch index.
constexpr int kMaxRanks = 8;
struct StoreMaps {
  CUtensorMap a[kMaxRanks];
  CUtensorMap b[kMaxRanks];
  int lq;          // channels per destination map
  int box_c;       // channels per TMA store (min(32, lq))
  int blk_base;    // outer coordinate offset (source rank * batch when scattering)
  int sys_fence;   // peers read the stores: fence at system scope before exiting
};

cudaError_t launch_input_stage(const CUtensorMap& zmap, const CUtensorMap& wmap,
                               const StoreMaps& smaps, const float* mask,
                               const float* u_in, const float* v_in, float2* zstats,
                               const PosTiling& tl, int incoming, int z_bf16, float eps, int* err,
                               int grid, cudaStream_t stream, int test_stall = 0);

cudaError_t launch_contraction(const CUtensorMap& amap, const CUtensorMap& bmap, __half* X, int L,
                               int M, int N, int K, int rows_per_block, int* err, int grid,
                               cudaStream_t stream);

// Scattered X rows: row block xb (its owner) starts at base[xb]; channel l of this
// launch is channel chan_off + l % lq of batch l / lq in the owner's (batch, c_total,
// rows, n) plane.
struct XDest {
  __half* base[kMaxRanks];
  int enabled, lq, c_total, chan_off;
};

// Layout of the CTA-pair contraction (fp16 elements). A and B are read through 5-D
// tensor maps (k in k block, row in row block, l, row block, k block); the kernel
// needs only the block sizes to form coordinates. X row i of channel l is stored at
// X + (i / x_rpb) * x_bs + l * x_ls + (i % x_rpb) * x_rs.
struct CtLayout {
  int a_rpb, b_rpb;   // rows per row block of A, B
  int k_rpb;          // k per k block (K when k is not split; a multiple of 64 otherwise)
  int x_rpb;          // rows per row block of X
  long long x_bs, x_ls, x_rs;
};

cudaError_t launch_contraction_pair(const CUtensorMap& amap, const CUtensorMap& bmap, __half* X,
                                    int L, int M, int N, int K, const CtLayout& lay, int* err,
                                    int num_sms, cudaStream_t stream,
                                    const XDest* xdest = nullptr, int a_mn = 0, int b_mn = 0);

cudaError_t launch_output_stage(const CUtensorMap& zmap, const CUtensorMap& xmap,
                                const CUtensorMap& wmap, const CUtensorMap& omap,
                                const float* mask, const float2* zstats, const float* u_g,
                                const float* v_g, const float* u_o, const float* v_o, void* out,
                                int out_dtype, const PosTiling& tl, int residual, int z_bf16,
                                float eps_in, float eps_out, int* err, int grid,
                                cudaStream_t stream);

// Argument checks of a whole square forward (ftm_trimul_fwd and the static-scratch
// entry): problem, rows == cols, non-null 16-byte-aligned z / packed / out / mask.
int check_forward_args(const ftm_problem* p, const void* z, const float* mask, const void* packed,
                       const void* out);
// What ftm_last_launch_count() reports for the calling thread.
void set_last_launch_count(int n);

cudaError_t launch_pack_params(const void* const params[16], int param_is_f16, int c_z, int c_h,
                               void* packed, cudaStream_t stream);

}  // namespace ftm
