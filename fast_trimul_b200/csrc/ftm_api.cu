// C ABI of fast_trimul_b200 (declared in include/fast_trimul_b200.h): argument
// checks, TMA tensor-map construction and the launch sequence of the three stages.
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <unordered_map>
#include <utility>

#include "../../include/fast_trimul_b200.h"
#include "ftm_kernels.h"

using namespace ftm;

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

thread_local int g_last_launches = 0;

int sm_count(int dev) {
  static int cache[64] = {0};
  int n = 0;
  if (dev >= 0 && dev < 64 && cache[dev]) {
    n = cache[dev];
  } else {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (dev >= 0 && dev < 64) cache[dev] = n;
  }
  // FTM_MAX_SMS caps the persistent grids (e.g. to leave SMs to a concurrent
  // communication kernel); read per call so a process can change it between calls
  const char* cap = getenv("FTM_MAX_SMS");
  if (cap) {
    const int c = atoi(cap);
    if (c >= 2 && c < n) n = c & ~1;
  }
  return n;
}

bool arch_ok(int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (dev_out) *dev_out = dev;
  return ftm_device_supported(dev) == 1;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// tiled map over `rank` dims (128B swizzle unless told otherwise); strides in bytes
// for dims 1..rank-1
// Encoding a tensor map costs microseconds of host time and a forward needs up to ~50 of
// them; identical requests (same device, base, shape, strides, box) are served from a
// bounded cache. A map holds no device state beyond the address it describes.
struct MapKey {
  int dev, dt, rank, swz;
  const void* base;
  uint64_t dims[5], strides[4];
  uint32_t box[5];
  bool operator==(const MapKey& o) const { return std::memcmp(this, &o, sizeof(MapKey)) == 0; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    const unsigned char* p = reinterpret_cast<const unsigned char*>(&k);
    uint64_t h = 1469598103934665603ull;
    for (size_t i = 0; i < sizeof(MapKey); ++i) h = (h ^ p[i]) * 1099511628211ull;
    return static_cast<size_t>(h);
  }
};

bool make_map(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base,
              const uint64_t* dims, const uint64_t* strides, const uint32_t* box,
              CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  MapKey key;
  std::memset(&key, 0, sizeof(key));
  if (cudaGetDevice(&key.dev) != cudaSuccess) return false;
  key.dt = static_cast<int>(dt);
  key.rank = rank;
  key.swz = static_cast<int>(swz);
  key.base = base;
  for (int i = 0; i < rank; ++i) {
    key.dims[i] = dims[i];
    key.box[i] = box[i];
  }
  for (int i = 0; i < rank - 1; ++i) key.strides[i] = strides[i];
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *m = it->second;
      return true;
    }
  }
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) s[i] = strides[i];
  const CUresult r =
      fn(m, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, b, e,
         CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() >= 1024) cache.clear();
  cache.emplace(key, *m);
  return true;
}

CUtensorMapDataType tma_dtype(int dt) {
  return dt == FTM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

int check_problem(const ftm_problem* p) {
  if (!p) return FTM_BAD_ARGUMENT;
  if (p->c_z != kC || p->c_h != kC) return FTM_BAD_SHAPE;
  if (p->batch < 1 || p->rows < 1 || p->cols < 1) return FTM_BAD_SHAPE;
  if (p->cols % 8 != 0) return FTM_BAD_SHAPE;  // TMA row strides must be 16-byte multiples
  if (p->mode != FTM_OUTGOING && p->mode != FTM_INCOMING) return FTM_BAD_ARGUMENT;
  // incoming mode writes the transposed planes (rows innermost): same 16-byte rule
  if (p->mode == FTM_INCOMING && p->rows % 8 != 0) return FTM_BAD_SHAPE;
  if (p->z_dtype != FTM_F16 && p->z_dtype != FTM_BF16) return FTM_BAD_DTYPE;
  if (p->out_dtype != FTM_F16 && p->out_dtype != FTM_BF16 && p->out_dtype != FTM_F32)
    return FTM_BAD_DTYPE;
  const double elems = double(p->batch) * p->rows * p->cols * kC;
  if (elems > 4.0e12) return FTM_BAD_SHAPE;
  return FTM_OK;
}

// z as (C, S, R, B) [natural] or (C, R, S, B) [incoming: consecutive tile rows walk r]
bool make_z_map(CUtensorMap* m, const ftm_problem* p, const void* z, bool transposed,
                const PosTiling& tl) {
  const uint64_t e = 2, C = kC, R = p->rows, S = p->cols, B = p->batch;
  uint64_t dims[4], strides[3];
  dims[0] = C;
  if (!transposed) {
    dims[1] = S; strides[0] = C * e;
    dims[2] = R; strides[1] = S * C * e;
  } else {
    dims[1] = R; strides[0] = S * C * e;
    dims[2] = S; strides[1] = C * e;
  }
  dims[3] = B;
  strides[2] = R * S * C * e;
  const uint32_t box[4] = {64, static_cast<uint32_t>(tl.vt), static_cast<uint32_t>(tl.ut), 1};
  return make_map(m, tma_dtype(p->z_dtype), 4, z, dims, strides, box);
}

// FTM_TEST_STALL=input makes the input stage withhold one tile load so its bounded
// waits expire: the failure-detection test of the device error path (no fault, no trap)
// L2 prefetch distance of a stage's producers in tiles: FTM_PREFETCH_IN / FTM_PREFETCH_OUT
// (or FTM_PREFETCH for both); the input stage gains from one tile ahead, the output stage
// (two streams already in flight per slot) from none
int prefetch_distance(const char* var, int dflt) {
  const char* v = getenv(var);
  if (!v || !*v) v = getenv("FTM_PREFETCH");
  if (!v || !*v) return dflt;
  const int d = atoi(v);
  return d < 0 ? 0 : (d > 8 ? 8 : d);
}

int test_stall_requested() {
  const char* v = getenv("FTM_TEST_STALL");
  return (v && strcmp(v, "input") == 0) ? 1 : 0;
}

// a_dst / b_dst null: a and b go to the local channel planes a_cm / b_cm (S, R, C, B).
// Otherwise each channel group goes to its owner rank's receive plane (see
// ftm_input_stage_scatter), one tensor map per destination.
int stage_in(const ftm_problem* p, const void* z, const float* mask, const void* packed,
             void* a_cm, void* b_cm, float* zstats, int* err, cudaStream_t stream, int dev,
             const ftm_peer_planes* a_dst = nullptr, const ftm_peer_planes* b_dst = nullptr) {
  // incoming: tiles run over (u = z column i, v = z row k), so a and b come out as the
  // transposed planes [c][i][k] the contraction reads K-major (k = z row)
  const bool incoming = p->mode == FTM_INCOMING;
  PosTiling tl;
  if (incoming) tl.init(p->batch, p->cols, p->rows);
  else tl.init(p->batch, p->rows, p->cols);
  tl.pf = prefetch_distance("FTM_PREFETCH_IN", 1);
  CUtensorMap zmap, wmap;
  if (!make_z_map(&zmap, p, z, incoming, tl)) return FTM_LAUNCH_FAILED;
  const PackedLayout L = PackedLayout::make(kC, kC);
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  {
    const uint64_t dims[2] = {kC, 4 * kC}, strides[1] = {kC * 2};
    const uint32_t box[2] = {64, 256};
    if (!make_map(&wmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, pk + L.w_in, dims, strides, box))
      return FTM_LAUNCH_FAILED;
  }
  // channel-major outputs: stores of [box_c channel x 64 position] blocks
  StoreMaps sm{};
  const uint64_t R = tl.R, S = tl.S, B = p->batch;   // planes (B, C, R, S), S innermost
  if (!a_dst) {
    sm.lq = kC;
    sm.box_c = 32;
    sm.blk_base = 0;
    sm.sys_fence = 0;
    const uint64_t dims[4] = {S, R, uint64_t(kC), B};
    const uint64_t strides[3] = {S * 2, R * S * 2, uint64_t(kC) * R * S * 2};
    const uint32_t box[4] = {64, 1, 32, 1};
    if (!make_map(&sm.a[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, a_cm, dims, strides, box) ||
        !make_map(&sm.b[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, b_cm, dims, strides, box))
      return FTM_LAUNCH_FAILED;
  } else {
    // receive plane of rank q: [source rank][batch][lq][rows][cols]
    const int P = a_dst->world, lq = kC / P;
    sm.lq = lq;
    sm.box_c = lq < 32 ? lq : 32;
    sm.blk_base = a_dst->rank * p->batch;
    sm.sys_fence = 1;
    const uint64_t dims[4] = {S, R, uint64_t(lq), uint64_t(P) * B};
    const uint64_t strides[3] = {S * 2, R * S * 2, uint64_t(lq) * R * S * 2};
    const uint32_t box[4] = {64, 1, uint32_t(sm.box_c), 1};
    for (int q = 0; q < P; ++q)
      if (!make_map(&sm.a[q], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, a_dst->base[q], dims, strides, box) ||
          !make_map(&sm.b[q], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, b_dst->base[q], dims, strides, box))
        return FTM_LAUNCH_FAILED;
  }
  const int grid = tl.tiles < sm_count(dev) ? tl.tiles : sm_count(dev);
  cudaError_t e = launch_input_stage(
      zmap, wmap, sm, mask, reinterpret_cast<const float*>(pk + L.u_in),
      reinterpret_cast<const float*>(pk + L.v_in), reinterpret_cast<float2*>(zstats), tl,
      incoming ? 1 : 0, p->z_dtype == FTM_BF16 ? 1 : 0, p->eps_in, err, grid, stream,
      test_stall_requested());
  return e == cudaSuccess ? FTM_OK : FTM_LAUNCH_FAILED;
}

// The CTA-pair kernel (256 x 256 tiles, ftm_contraction2.cu) is the default; the
// single-CTA kernel (128 x 256 tiles) is kept for comparison: FTM_CONTRACTION=single.
bool use_pair_contraction() {
  const char* v = getenv("FTM_CONTRACTION");
  return !(v && strcmp(v, "single") == 0);
}

// 5-D operand map (k in k block, row in row block, l, row block, k block) of one
// contraction operand; strides in elements. A single row / k block gets a stride that
// spans everything before it.
bool make_operand_map(CUtensorMap* m, const void* base, int L, int rows, int rpb, int k, int kpb,
                      long long bs, long long ls, long long rs, long long kbs) {
  const uint64_t nrb = uint64_t((rows + rpb - 1) / rpb), nkb = uint64_t(k / kpb);
  if (nrb == 1) bs = ls * L;
  if (nkb == 1) kbs = bs * static_cast<long long>(nrb);
  const uint64_t dims[5] = {uint64_t(kpb), uint64_t(rpb), uint64_t(L), nrb, nkb};
  const uint64_t strides[4] = {uint64_t(rs) * 2, uint64_t(ls) * 2, uint64_t(bs) * 2, uint64_t(kbs) * 2};
  const uint32_t box[5] = {kCtBK, 128u, 1, 1, 1};
  return make_map(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, base, dims, strides, box);
}

// MN-major operand map: (row, k, l, 1, 1) with rows contiguous and k rows `rs` apart;
// 64 x 64 boxes (two per 128-row half).
bool make_operand_map_mn(CUtensorMap* m, const void* base, int L, int rows, int k, long long ls,
                         long long rs) {
  const uint64_t dims[5] = {uint64_t(rows), uint64_t(k), uint64_t(L), 1, 1};
  const uint64_t strides[4] = {uint64_t(rs) * 2, uint64_t(ls) * 2, uint64_t(ls) * 2 * L,
                               uint64_t(ls) * 2 * L};
  const uint32_t box[5] = {64u, uint32_t(kCtBK), 1, 1, 1};
  return make_map(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, base, dims, strides, box);
}

// Checks of a general layout (see ftm_contraction_layout); normalises single-block
// sizes. Returns an ftm_status.
int check_layout(ftm_contraction_layout* d) {
  if (!d || !d->a || !d->b || !d->x) return FTM_BAD_ARGUMENT;
  if (d->L < 1 || d->m < 1 || d->n < 1 || d->k < 1) return FTM_BAD_SHAPE;
  if (d->n % 8 != 0) return FTM_BAD_SHAPE;
  if (d->k_per_block <= 0 || d->k_per_block >= d->k) d->k_per_block = d->k;
  if (d->k_per_block < d->k && (d->k % d->k_per_block != 0 || d->k_per_block % kCtBK != 0))
    return FTM_BAD_SHAPE;
  if (d->a_rows_per_block <= 0 || d->a_rows_per_block >= d->m) d->a_rows_per_block = d->m;
  else if (d->m % d->a_rows_per_block != 0 || d->a_rows_per_block % 128 != 0) return FTM_BAD_SHAPE;
  if (d->b_rows_per_block <= 0 || d->b_rows_per_block >= d->n) d->b_rows_per_block = d->n;
  else if (d->n % d->b_rows_per_block != 0 || d->b_rows_per_block % 128 != 0) return FTM_BAD_SHAPE;
  if (d->x_rows_per_block <= 0 || d->x_rows_per_block >= d->m) d->x_rows_per_block = d->m;
  else if (d->m % d->x_rows_per_block != 0) return FTM_BAD_SHAPE;
  const long long strides[] = {d->a_l_stride, d->a_row_stride, d->b_l_stride, d->b_row_stride,
                               d->x_l_stride, d->x_row_stride};
  for (long long s : strides)
    if (s <= 0 || s % 8 != 0) return FTM_BAD_ALIGN;
  const long long opt[] = {d->a_block_stride, d->a_kblock_stride, d->b_block_stride,
                           d->b_kblock_stride, d->x_block_stride};
  for (long long s : opt)
    if (s < 0 || s % 8 != 0) return FTM_BAD_ALIGN;
  if (d->a_mn_major || d->b_mn_major) {
    // MN-major operands: one row block, one k block, rows contiguous
    if (d->k_per_block != d->k) return FTM_BAD_SHAPE;
    if (d->a_mn_major && (d->a_rows_per_block != d->m || d->a_row_stride < d->m)) return FTM_BAD_SHAPE;
    if (d->b_mn_major && (d->b_rows_per_block != d->n || d->b_row_stride < d->n)) return FTM_BAD_SHAPE;
  }
  if ((!d->a_mn_major && d->a_row_stride < d->k_per_block) ||
      (!d->b_mn_major && d->b_row_stride < d->k_per_block))
    return FTM_BAD_SHAPE;
  if (!aligned16(d->a) || !aligned16(d->b) || !aligned16(d->x)) return FTM_BAD_ALIGN;
  return FTM_OK;
}

int stage_contract_general(const ftm_contraction_layout& d, int* err, cudaStream_t stream, int dev,
                           const XDest* xdest = nullptr) {
  CUtensorMap amap, bmap;
  const bool a_ok = d.a_mn_major
                        ? make_operand_map_mn(&amap, d.a, d.L, d.m, d.k, d.a_l_stride, d.a_row_stride)
                        : make_operand_map(&amap, d.a, d.L, d.m, d.a_rows_per_block, d.k, d.k_per_block,
                                           d.a_block_stride, d.a_l_stride, d.a_row_stride,
                                           d.a_kblock_stride);
  const bool b_ok = d.b_mn_major
                        ? make_operand_map_mn(&bmap, d.b, d.L, d.n, d.k, d.b_l_stride, d.b_row_stride)
                        : make_operand_map(&bmap, d.b, d.L, d.n, d.b_rows_per_block, d.k, d.k_per_block,
                                           d.b_block_stride, d.b_l_stride, d.b_row_stride,
                                           d.b_kblock_stride);
  if (!a_ok || !b_ok) return FTM_LAUNCH_FAILED;
  CtLayout lay{d.a_rows_per_block, d.b_rows_per_block, d.k_per_block, d.x_rows_per_block,
               d.x_block_stride, d.x_l_stride, d.x_row_stride};
  const cudaError_t e = launch_contraction_pair(amap, bmap, static_cast<__half*>(d.x), d.L, d.m,
                                                d.n, d.k, lay, err, sm_count(dev), stream, xdest,
                                                d.a_mn_major ? 1 : 0, d.b_mn_major ? 1 : 0);
  return e == cudaSuccess ? FTM_OK : FTM_LAUNCH_FAILED;
}

// A (and X) as a_blocks row blocks of (L, a_rpb, k), B as `blocks` row blocks of
// (L, rpb, k): the layouts of ftm_contraction_blocked.
ftm_contraction_layout blocked_layout(const void* A, const void* B, void* X, int L, int a_rpb,
                                      int a_blocks, int k, int rpb, int blocks) {
  ftm_contraction_layout d{};
  const long long m = static_cast<long long>(a_rpb) * a_blocks, n = static_cast<long long>(rpb) * blocks;
  d.L = L; d.m = static_cast<int>(m); d.n = static_cast<int>(n); d.k = k; d.k_per_block = k;
  d.a = A; d.a_rows_per_block = a_rpb;
  d.a_row_stride = k; d.a_l_stride = static_cast<long long>(a_rpb) * k;
  d.a_block_stride = d.a_l_stride * L;
  d.b = B; d.b_rows_per_block = rpb;
  d.b_row_stride = k; d.b_l_stride = static_cast<long long>(rpb) * k;
  d.b_block_stride = d.b_l_stride * L;
  d.x = X; d.x_rows_per_block = a_rpb;
  d.x_row_stride = n; d.x_l_stride = a_rpb * n; d.x_block_stride = d.x_l_stride * L;
  return d;
}

int stage_contract(const void* A, const void* B, void* X, int L, int a_rpb, int a_blocks, int k,
                   int rpb, int blocks, int* err, cudaStream_t stream, int dev,
                   const XDest* xdest = nullptr) {
  // the single-CTA kernel reads B in 256-row tiles: blocked B of 128-row blocks and
  // blocked A always go to the pair kernel
  const bool pair = use_pair_contraction() || a_blocks > 1 || xdest != nullptr ||
                    (blocks > 1 && rpb % kCtBN != 0);
  const int m = a_rpb * a_blocks;
  const int n = rpb * blocks;
  if (pair) {
    ftm_contraction_layout d = blocked_layout(A, B, X, L, a_rpb, a_blocks, k, rpb, blocks);
    const int st = check_layout(&d);
    if (st != FTM_OK) return st;
    return stage_contract_general(d, err, stream, dev, xdest);
  }
  CUtensorMap amap, bmap;
  {
    const uint64_t dims[3] = {uint64_t(k), uint64_t(m), uint64_t(L)};
    const uint64_t strides[2] = {uint64_t(k) * 2, uint64_t(m) * k * 2};
    const uint32_t box[3] = {kCtBK, kCtBM, 1};
    if (!make_map(&amap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, A, dims, strides, box))
      return FTM_LAUNCH_FAILED;
  }
  {
    const uint64_t dims[4] = {uint64_t(k), uint64_t(rpb), uint64_t(L), uint64_t(blocks)};
    const uint64_t strides[3] = {uint64_t(k) * 2, uint64_t(rpb) * k * 2,
                                 uint64_t(L) * rpb * k * 2};
    const uint32_t box[4] = {kCtBK, uint32_t(kCtBN), 1, 1};
    if (!make_map(&bmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, B, dims, strides, box))
      return FTM_LAUNCH_FAILED;
  }
  const long tiles = long(L) * ((m + kCtBM - 1) / kCtBM) * ((n + kCtBN - 1) / kCtBN);
  const int grid = tiles < sm_count(dev) ? int(tiles) : sm_count(dev);
  const cudaError_t e =
      launch_contraction(amap, bmap, static_cast<__half*>(X), L, m, n, k, rpb, err, grid, stream);
  return e == cudaSuccess ? FTM_OK : FTM_LAUNCH_FAILED;
}

// Contraction whose reduction index is split into k_blocks blocks of k_rpb (A, B stored
// [k block][L][m or n][k_rpb] -- the channel-shard layout of the incoming transposed
// planes), X written as (m / x_rpb) blocks of (L, x_rpb, n), or scattered to owners.
int stage_contract_kblocked(const void* A, const void* B, void* X, int L, int m, int n, int k_rpb,
                            int k_blocks, int x_rpb, int* err, cudaStream_t stream, int dev,
                            const XDest* xdest = nullptr) {
  ftm_contraction_layout d{};
  d.L = L; d.m = m; d.n = n; d.k = k_rpb * k_blocks; d.k_per_block = k_rpb;
  d.a = A; d.a_rows_per_block = m; d.a_row_stride = k_rpb;
  d.a_l_stride = static_cast<long long>(m) * k_rpb; d.a_kblock_stride = d.a_l_stride * L;
  d.b = B; d.b_rows_per_block = n; d.b_row_stride = k_rpb;
  d.b_l_stride = static_cast<long long>(n) * k_rpb; d.b_kblock_stride = d.b_l_stride * L;
  d.x = X; d.x_rows_per_block = x_rpb; d.x_row_stride = n;
  d.x_l_stride = static_cast<long long>(x_rpb) * n; d.x_block_stride = d.x_l_stride * L;
  const int st = check_layout(&d);
  if (st != FTM_OK) return st;
  return stage_contract_general(d, err, stream, dev, xdest);
}

int stage_out(const ftm_problem* p, const void* z, const float* mask, const void* x_cm,
              const float* zstats, const void* packed, void* out, int* err, cudaStream_t stream,
              int dev) {
  PosTiling tl;
  tl.init(p->batch, p->rows, p->cols);
  tl.pf = prefetch_distance("FTM_PREFETCH_OUT", 0);
  CUtensorMap zmap, xmap, wmap;
  if (!make_z_map(&zmap, p, z, false, tl)) return FTM_LAUNCH_FAILED;
  {
    const uint64_t R = p->rows, S = p->cols;
    const uint64_t dims[4] = {S, R, uint64_t(kC), uint64_t(p->batch)};
    const uint64_t strides[3] = {S * 2, R * S * 2, uint64_t(kC) * R * S * 2};
    const uint32_t box[4] = {64, 1, kC, 1};
    if (!make_map(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, x_cm, dims, strides, box))
      return FTM_LAUNCH_FAILED;
  }
  const PackedLayout L = PackedLayout::make(kC, kC);
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  {
    const uint64_t dims[2] = {kC, 2 * kC}, strides[1] = {kC * 2};
    const uint32_t box[2] = {64, 256};
    if (!make_map(&wmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, pk + L.w_out, dims, strides, box))
      return FTM_LAUNCH_FAILED;
  }
  const int grid = tl.tiles < sm_count(dev) ? tl.tiles : sm_count(dev);
  // out (16-bit) written like z: (C, S, R, B), 32 positions x 64 channels per store
  CUtensorMap omap = zmap;
  if (p->out_dtype != FTM_F32) {
    const uint64_t C = kC, R = p->rows, S = p->cols, B = p->batch;
    const uint64_t dims[4] = {C, S, R, B};
    const uint64_t strides[3] = {C * 2, S * C * 2, R * S * C * 2};
    const uint32_t box[4] = {64, 32, 1, 1};
    if (!make_map(&omap, tma_dtype(p->out_dtype), 4, out, dims, strides, box))
      return FTM_LAUNCH_FAILED;
  }
  cudaError_t e = launch_output_stage(
      zmap, xmap, wmap, omap, mask, reinterpret_cast<const float2*>(zstats),
      reinterpret_cast<const float*>(pk + L.u_g),
      reinterpret_cast<const float*>(pk + L.v_g), reinterpret_cast<const float*>(pk + L.u_o),
      reinterpret_cast<const float*>(pk + L.v_o), out, p->out_dtype, tl, p->residual ? 1 : 0,
      p->z_dtype == FTM_BF16 ? 1 : 0, p->eps_in, p->eps_out, err, grid, stream);
  return e == cudaSuccess ? FTM_OK : FTM_LAUNCH_FAILED;
}

struct WsLayout {
  size_t a, b, x, stats, err, total;
};

WsLayout ws_layout(const ftm_problem* p) {
  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  const size_t plane = size_t(p->batch) * kC * p->rows * p->cols * 2;
  WsLayout w{};
  w.a = 0;
  w.b = up(plane);
  w.x = w.b + up(plane);
  w.stats = w.x + up(plane);
  w.err = w.stats + up(size_t(p->batch) * p->rows * p->cols * 8);
  w.total = w.err + 256;
  return w;
}

}  // namespace

namespace ftm {

cudaError_t set_smem_once(const void* kern, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({kern, dev})) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.insert({kern, dev});
  return e;
}

bool pdl_enabled() {
  const char* v = getenv("FTM_PDL");
  return !(v && strcmp(v, "0") == 0);
}

int check_forward_args(const ftm_problem* p, const void* z, const float* mask, const void* packed,
                       const void* out) {
  const int st = check_problem(p);
  if (st != FTM_OK) return st;
  if (p->rows != p->cols) return FTM_BAD_SHAPE;  // row shards go through the stage calls
  if (!z || !packed || !out) return FTM_BAD_ARGUMENT;
  if (!aligned16(z) || !aligned16(packed) || !aligned16(out) || (mask && !aligned16(mask)))
    return FTM_BAD_ALIGN;
  return FTM_OK;
}

void set_last_launch_count(int n) { g_last_launches = n; }

}  // namespace ftm

extern "C" {

size_t ftm_packed_params_bytes(int32_t c_z, int32_t c_h) {
  return PackedLayout::make(c_z, c_h).total;
}

int ftm_pack_params(const void* const params[16], int32_t param_dtype, int32_t c_z, int32_t c_h,
                    void* packed, ftm_stream_t stream) {
  g_last_launches = 0;
  if (!params || !packed) return FTM_BAD_ARGUMENT;
  for (int i = 0; i < 16; ++i)
    if (!params[i]) return FTM_BAD_ARGUMENT;
  if (param_dtype != FTM_F16 && param_dtype != FTM_F32) return FTM_BAD_DTYPE;
  if (c_z < 1 || c_h < 1 || c_z > 4096 || c_h > 4096) return FTM_BAD_SHAPE;
  if (!aligned16(packed)) return FTM_BAD_ALIGN;
  int dev;
  if (!arch_ok(&dev)) return FTM_UNSUPPORTED_ARCH;
  cudaError_t e = launch_pack_params(params, param_dtype == FTM_F16 ? 1 : 0, c_z, c_h, packed,
                                     reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return FTM_LAUNCH_FAILED;
  g_last_launches = 1;
  return FTM_OK;
}

size_t ftm_workspace_bytes(const ftm_problem* p) {
  if (check_problem(p) != FTM_OK) return 0;
  return ws_layout(p).total;
}

int* ftm_workspace_error_word(const ftm_problem* p, void* workspace) {
  if (!workspace || check_problem(p) != FTM_OK) return nullptr;
  return reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + ws_layout(p).err);
}

int ftm_trimul_fwd(const ftm_problem* p, const void* z, const float* mask, const void* packed,
                   void* out, void* workspace, size_t workspace_bytes, ftm_stream_t stream) {
  g_last_launches = 0;
  int st = check_forward_args(p, z, mask, packed, out);
  if (st != FTM_OK) return st;
  const WsLayout w = ws_layout(p);
  if (!workspace || workspace_bytes < w.total) return FTM_BAD_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255u) return FTM_BAD_ALIGN;
  int dev;
  if (!arch_ok(&dev)) return FTM_UNSUPPORTED_ARCH;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* err = reinterpret_cast<int*>(ws + w.err);
  if (cudaMemsetAsync(err, 0, sizeof(int), s) != cudaSuccess) return FTM_LAUNCH_FAILED;
  const int N = p->cols, L = p->batch * kC;
  float* zst = reinterpret_cast<float*>(ws + w.stats);
  if ((st = stage_in(p, z, mask, packed, ws + w.a, ws + w.b, zst, err, s, dev)) != FTM_OK) return st;
  if ((st = stage_contract(ws + w.a, ws + w.b, ws + w.x, L, N, 1, N, N, 1, err, s, dev)) != FTM_OK)
    return st;
  if ((st = stage_out(p, z, mask, ws + w.x, zst, packed, out, err, s, dev)) != FTM_OK) return st;
  g_last_launches = 3;
  return FTM_OK;
}

int ftm_input_stage(const ftm_problem* p, const void* z, const float* mask, const void* packed,
                    void* a_cm, void* b_cm, float* zstats, int* err_word, ftm_stream_t stream) {
  g_last_launches = 0;
  int st = check_problem(p);
  if (st != FTM_OK) return st;
  if (!z || !packed || !a_cm || !b_cm || !zstats || !err_word) return FTM_BAD_ARGUMENT;
  if (!aligned16(z) || !aligned16(packed) || !aligned16(a_cm) || !aligned16(b_cm) ||
      (mask && !aligned16(mask)))
    return FTM_BAD_ALIGN;
  int dev;
  if (!arch_ok(&dev)) return FTM_UNSUPPORTED_ARCH;
  st = stage_in(p, z, mask, packed, a_cm, b_cm, zstats, err_word,
                reinterpret_cast<cudaStream_t>(stream), dev);
  if (st == FTM_OK) g_last_launches = 1;
  return st;
}

int ftm_contraction(const void* A, const void* B, void* X, int32_t L, int32_t m, int32_t k,
                    int32_t b_rows_per_block, int32_t b_blocks, int* err_word,
                    ftm_stream_t stream) {
  return ftm_contraction_blocked(A, B, X, L, m, 1, k, b_rows_per_block, b_blocks, err_word, stream);
}

int ftm_contraction_blocked(const void* A, const void* B, void* X, int32_t L,
                            int32_t a_rows_per_block, int32_t a_blocks, int32_t k,
                            int32_t b_rows_per_block, int32_t b_blocks, int* err_word,
                            ftm_stream_t stream) {
  g_last_launches = 0;
  if (!A || !B || !X || !err_word) return FTM_BAD_ARGUMENT;
  if (L < 1 || a_rows_per_block < 1 || a_blocks < 1 || k < 1 || b_rows_per_block < 1 ||
      b_blocks < 1)
    return FTM_BAD_SHAPE;
  if (k % 8 != 0 || (b_rows_per_block * b_blocks) % 8 != 0) return FTM_BAD_SHAPE;
  if (b_blocks > 1 && b_rows_per_block % 128 != 0) return FTM_BAD_SHAPE;
  if (a_blocks > 1 && a_rows_per_block % kCtBM != 0) return FTM_BAD_SHAPE;
  if (!aligned16(A) || !aligned16(B) || !aligned16(X)) return FTM_BAD_ALIGN;
  int dev;
  if (!arch_ok(&dev)) return FTM_UNSUPPORTED_ARCH;
  const int st = stage_contract(A, B, X, L, a_rows_per_block, a_blocks, k, b_rows_per_block,
                                b_blocks, err_word, reinterpret_cast<cudaStream_t>(stream), dev);
  if (st == FTM_OK) g_last_launches = 1;
  return st;
}

static bool peers_ok(const ftm_peer_planes* d) {
  if (!d || d->world < 1 || d->world > FTM_MAX_RANKS || d->rank < 0 || d->rank >= d->world)
    return false;
  if (kC % d->world != 0 || (kC / d->world) % 16 != 0) return false;
  for (int q = 0; q < d->world; ++q)
    if (!d->base[q] || !aligned16(d->base[q])) return false;
  return true;
}

int ftm_input_stage_scatter(const ftm_problem* p, const void* z, const float* mask,
                            const void* packed, const ftm_peer_planes* a_dst,
                            const ftm_peer_planes* b_dst, float* zstats, int* err_word,
                            ftm_stream_t stream) {
  g_last_launches = 0;
  int st = check_problem(p);
  if (st != FTM_OK) return st;
  if (!z || !packed || !zstats || !err_word || !a_dst || !b_dst) return FTM_BAD_ARGUMENT;
  if (!peers_ok(a_dst) || !peers_ok(b_dst) || a_dst->world != b_dst->world ||
      a_dst->rank != b_dst->rank)
    return FTM_BAD_ARGUMENT;
  if (!aligned16(z) || !aligned16(packed) || (mask && !aligned16(mask))) return FTM_BAD_ALIGN;
  int dev;
  if (!arch_ok(&dev)) return FTM_UNSUPPORTED_ARCH;
  st = stage_in(p, z, mask, packed, nullptr, nullptr, zstats, err_word,
                reinterpret_cast<cudaStream_t>(stream), dev, a_dst, b_dst);
  if (st == FTM_OK) g_last_launches = 1;
  return st;
}

int ftm_contraction_scatter(const void* A, const void* B, const ftm_peer_planes* x_dst,
                            int32_t batch, int32_t c_h, int32_t rows, int32_t n, int32_t mode,
                            int* err_word, ftm_stream_t stream) {
  g_last_launches = 0;
  if (!A || !B || !err_word || !x_dst) return FTM_BAD_ARGUMENT;
  if (c_h != kC || !peers_ok(x_dst)) return FTM_BAD_ARGUMENT;
  if (mode != FTM_OUTGOING && mode != FTM_INCOMING) return FTM_BAD_ARGUMENT;
  const int P = x_dst->world, lq = kC / P;
  if (batch < 1 || rows < 1 || n != P * rows || rows % kCtBN != 0) return FTM_BAD_SHAPE;
  if (!aligned16(A) || !aligned16(B)) return FTM_BAD_ALIGN;
  int dev;
  if (!arch_ok(&dev)) return FTM_UNSUPPORTED_ARCH;
  XDest xd{};
  for (int q = 0; q < P; ++q) xd.base[q] = static_cast<__half*>(x_dst->base[q]);
  xd.enabled = 1;
  xd.lq = lq;
  xd.c_total = kC;
  xd.chan_off = x_dst->rank * lq;
  // outgoing: A, B are P row blocks (one per source rank) of (batch * lq, rows, n);
  // incoming: P blocks of the transposed planes (batch * lq, n, rows) -- k split by rank
  const int st =
      mode == FTM_OUTGOING
          ? stage_contract(A, B, x_dst->base[x_dst->rank], batch * lq, rows, P, n, rows, P, err_word,
                           reinterpret_cast<cudaStream_t>(stream), dev, &xd)
          : stage_contract_kblocked(A, B, x_dst->base[x_dst->rank], batch * lq, n, n, rows, P, rows,
                                    err_word, reinterpret_cast<cudaStream_t>(stream), dev, &xd);
  if (st == FTM_OK) g_last_launches = 1;
  return st;
}

int ftm_contraction_kblocked(const void* A, const void* B, void* X, int32_t L, int32_t m,
                             int32_t n, int32_t k_rows_per_block, int32_t k_blocks,
                             int32_t x_rows_per_block, int* err_word, ftm_stream_t stream) {
  g_last_launches = 0;
  if (!A || !B || !X || !err_word) return FTM_BAD_ARGUMENT;
  if (L < 1 || m < 1 || n < 1 || k_rows_per_block < 1 || k_blocks < 1 || x_rows_per_block < 1)
    return FTM_BAD_SHAPE;
  if (k_rows_per_block % kCtBK != 0 || m % x_rows_per_block != 0 || n % 8 != 0 ||
      (m / x_rows_per_block > 1 && x_rows_per_block % kCtBN != 0))
    return FTM_BAD_SHAPE;
  if (!aligned16(A) || !aligned16(B) || !aligned16(X)) return FTM_BAD_ALIGN;
  int dev;
  if (!arch_ok(&dev)) return FTM_UNSUPPORTED_ARCH;
  const int st = stage_contract_kblocked(A, B, X, L, m, n, k_rows_per_block, k_blocks,
                                         x_rows_per_block, err_word,
                                         reinterpret_cast<cudaStream_t>(stream), dev);
  if (st == FTM_OK) g_last_launches = 1;
  return st;
}

int ftm_contraction_general(const ftm_contraction_layout* layout, int* err_word,
                            ftm_stream_t stream) {
  g_last_launches = 0;
  if (!layout || !err_word) return FTM_BAD_ARGUMENT;
  ftm_contraction_layout d = *layout;
  int st = check_layout(&d);
  if (st != FTM_OK) return st;
  int dev;
  if (!arch_ok(&dev)) return FTM_UNSUPPORTED_ARCH;
  st = stage_contract_general(d, err_word, reinterpret_cast<cudaStream_t>(stream), dev);
  if (st == FTM_OK) g_last_launches = 1;
  return st;
}

int ftm_output_stage(const ftm_problem* p, const void* z, const float* mask, const void* x_cm,
                     const float* zstats, const void* packed, void* out, int* err_word,
                     ftm_stream_t stream) {
  g_last_launches = 0;
  int st = check_problem(p);
  if (st != FTM_OK) return st;
  if (!z || !x_cm || !zstats || !packed || !out || !err_word) return FTM_BAD_ARGUMENT;
  if (!aligned16(z) || !aligned16(x_cm) || !aligned16(packed) || !aligned16(out) ||
      (mask && !aligned16(mask)))
    return FTM_BAD_ALIGN;
  int dev;
  if (!arch_ok(&dev)) return FTM_UNSUPPORTED_ARCH;
  st = stage_out(p, z, mask, x_cm, zstats, packed, out, err_word,
                 reinterpret_cast<cudaStream_t>(stream), dev);
  if (st == FTM_OK) g_last_launches = 1;
  return st;
}

int ftm_check_error(const int* err_word, int* detail, ftm_stream_t stream) {
  if (!err_word) return FTM_BAD_ARGUMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(s) != cudaSuccess) return FTM_LAUNCH_FAILED;
  int v = 0;
  if (cudaMemcpy(&v, err_word, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return FTM_LAUNCH_FAILED;
  if (detail) *detail = v;
  if (v != 0) {
    cudaMemset(const_cast<int*>(err_word), 0, sizeof(int));
    return FTM_TIMEOUT;
  }
  return FTM_OK;
}

const char* ftm_status_string(int status) {
  switch (status) {
    case FTM_OK: return "ok";
    case FTM_BAD_SHAPE: return "unsupported shape (needs c_z == c_h == 128, N % 8 == 0)";
    case FTM_BAD_DTYPE: return "unsupported dtype";
    case FTM_BAD_ALIGN: return "pointer not 16-byte aligned (workspace: 256-byte)";
    case FTM_UNSUPPORTED_ARCH: return "device is not an sm_100 (B200-class) GPU";
    case FTM_LAUNCH_FAILED: return "kernel launch or tensor-map encoding failed";
    case FTM_TIMEOUT: return "a bounded device-side wait expired";
    case FTM_BAD_WORKSPACE: return "workspace missing or too small";
    case FTM_BAD_ARGUMENT: return "invalid argument";
    default: return "unknown status";
  }
}

int ftm_device_supported(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess)
    return 0;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess)
    return 0;
  return (major == 10 && minor == 0) ? 1 : 0;
}

int ftm_last_launch_count(void) { return g_last_launches; }

}  // extern "C"
