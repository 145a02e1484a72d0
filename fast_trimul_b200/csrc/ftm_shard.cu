// Row-sharded multi-GPU forward: the native pipeline behind ftm_shard_forward.
//
// Rank r owns R = N / P consecutive rows of z (and of the output). The input stage runs
// on the local rows in `row_chunks` launches; as each chunk finishes, the copy engines
// push its pieces to the ranks that need them, straight into their receive windows over
// NVLink (CUDA IPC mappings), and a one-thread kernel on the same copy stream raises a
// flag word in the receiver's memory. Receivers wait for their flags with a bounded
// device-side wait kernel -- no NCCL call and no host synchronisation on the data path.
//
//   alltoall (both modes): chunk r's channel shard q (128 / P channels) goes to rank q.
//     Rank q contracts its channels over all N rows, one row owner at a time (owner
//     me + 1 first, itself last), and the x block of each owner is pushed back to that
//     owner's x plane as soon as it is done. Bytes each rank sends per forward:
//     3 (P - 1) / P^2 of the full a/b/x plane.
//   allgather (outgoing): chunk r's b goes to every rank; each rank contracts its own
//     rows against its own b at once and against each arriving chunk of a peer's b.
//     Bytes sent: (P - 1) / P of the b plane; fewer than alltoall at P = 2.
//
// Buffer reuse across forwards (no extra barrier): receive windows are double-buffered
// by forward parity. A rank pushes forward t + 1 into a peer's slot only after its own
// output stage of forward t, which waited for data that the peer produced after all of
// its forward t - 1 work, so the slot of t - 1 is no longer read. x planes and local
// buffers are ordered by events between the compute and copy streams. Flags carry the
// forward's epoch (monotonic), so they never need resetting.
//
// Every wait is bounded (FTM_SHARD_WAIT_NS); an expired wait records
// (KERNEL_EXCHANGE << 8) | (kind << 4) | 1 in the error word and lets the forward run on
// (its output is then invalid; the caller reads the word with ftm_check_error).
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>

#include "../../include/fast_trimul_b200.h"
#include "ftm_kernels.h"

#ifndef FTM_SHARD_WAIT_NS
#define FTM_SHARD_WAIT_NS 20000000000ull  // 20 s: ranks may start a forward seconds apart
#endif

namespace ftm {
namespace {

constexpr int KERNEL_EXCHANGE = 5;
constexpr int kFlagAB = 0;                       // [src][chunk] a/b (or b) arrived
constexpr int kFlagX = FTM_MAX_RANKS * FTM_SHARD_MAX_ROW_CHUNKS;   // [src] x block arrived

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until flags[idx[i]] >= epoch for every i < count (one warp, bounded).
struct FlagList {
  int idx[FTM_MAX_RANKS * FTM_SHARD_MAX_ROW_CHUNKS];
  int count;
};

__global__ void wait_flags_kernel(const int* flags, const FlagList list, int epoch, int* err,
                                  int code) {
  const uint64_t t0 = globaltimer_ns();
  bool ok = true;
  for (int i = threadIdx.x; ok && i < list.count; i += 32) {
    const int* f = flags + list.idx[i];
    while (ld_acquire_sys(f) < epoch) {
      if (globaltimer_ns() - t0 > FTM_SHARD_WAIT_NS) {
        atomicCAS(err, 0, code);
        ok = false;
        break;
      }
      __nanosleep(256);
    }
  }
  __syncwarp();
  __threadfence();
}

// Raise one flag word (usually in a peer's memory) to `epoch`, after everything queued
// before this launch on its stream -- the copies it announces -- has completed.
__global__ void signal_kernel(int* flag, int epoch) {
  __threadfence_system();
  st_release_sys(flag, epoch);
}

// SM-driven push: copies up to kMaxSegs (src, dst) runs of 16-byte words -- dst usually
// in a peer's memory -- with every CTA taking a strided share of each run, four words in
// flight per thread. With `nflags` > 0 the last CTA to finish raises each flag to
// `epoch` after all CTAs' stores are fenced at system scope.
constexpr int kMaxSegs = 64;
struct PushList {
  const uint4* src[kMaxSegs];
  uint4* dst[kMaxSegs];
  unsigned long long n16[kMaxSegs];
  int* flag[FTM_MAX_RANKS];
  int count, nflags, epoch;
  unsigned int* done;   // CTA counter (zero between launches)
};

__global__ void __launch_bounds__(256) push_kernel(const __grid_constant__ PushList pl) {
  const unsigned long long stride = static_cast<unsigned long long>(gridDim.x) * blockDim.x;
  const unsigned long long t0 = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int s = 0; s < pl.count; ++s) {
    const uint4* __restrict__ src = pl.src[s];
    uint4* dst = pl.dst[s];
    const unsigned long long n = pl.n16[s];
    unsigned long long i = t0;
    for (; i + 3 * stride < n; i += 4 * stride) {
      const uint4 v0 = __ldg(src + i), v1 = __ldg(src + i + stride);
      const uint4 v2 = __ldg(src + i + 2 * stride), v3 = __ldg(src + i + 3 * stride);
      dst[i] = v0;
      dst[i + stride] = v1;
      dst[i + 2 * stride] = v2;
      dst[i + 3 * stride] = v3;
    }
    for (; i < n; i += stride) dst[i] = __ldg(src + i);
  }
  if (pl.nflags == 0) return;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(pl.done, 1u) == gridDim.x - 1) {
      __threadfence_system();
      for (int f = 0; f < pl.nflags; ++f) st_release_sys(pl.flag[f], pl.epoch);
      *pl.done = 0;
    }
  }
}

// Trace point (only when a trace buffer is configured): records the device clock when
// everything queued before it on its stream has finished.
__global__ void mark_kernel(long long* trace, int slot, int tag) {
  trace[2 * slot] = static_cast<long long>(globaltimer_ns());
  trace[2 * slot + 1] = tag;
}

}  // namespace
}  // namespace ftm

using namespace ftm;

struct ftm_shard_plan {
  ftm_shard_config cfg;
  int P, me, RC, rc, R, N, B, L, lq, dev;
  size_t unit;              // fp16 elements of one channel of one chunk (rc * N)
  cudaStream_t copy;        // a/b pushes and their signals
  cudaStream_t copy_x;      // x pushes and their signals: a forward's x pushes and the next
                            // forward's a/b pushes must not queue behind each other
  cudaStream_t cur;         // the one of the two the current pushes go to
  cudaEvent_t ev_in[FTM_SHARD_MAX_ROW_CHUNKS];
  cudaEvent_t ev_owner[FTM_MAX_RANKS];
  cudaEvent_t ev_pushed;    // last forward's a/b pushes done reading the local planes
  cudaEvent_t ev_x_pushed;  // last forward's x pushes done reading the x blocks
  int epoch;
  int launches;             // kernels launched by the current forward
  long long* trace;         // optional (time, tag) pairs of the current forward
  int trace_n;
  ftm_problem out_problem;  // the shard problem with this forward's output dtype
  int sm_push;              // pushes by push_kernel (FTM_SHARD_PUSH=sm) instead of copy engines
  int push_ctas;
  unsigned int* push_done;  // counters for push_kernel, one per copy stream
  PushList pending;         // runs queued for the next push
  // FTM_SHARD_HOSTPROF=1: host time spent issuing each kind of work, printed at destroy
  int hostprof;
  double host_ns[8];
  long long forwards;
};

namespace {
enum { H_INPUT, H_CONTRACT, H_COPY, H_SIGNAL, H_WAIT, H_OUTPUT, H_TOTAL, H_COUNT };
const char* const kHostNames[H_COUNT] = {"input stage", "contraction", "copies", "signals",
                                         "waits", "output stage", "whole forward"};
struct HostTimer {
  ftm_shard_plan* pl;
  int cat;
  std::chrono::steady_clock::time_point t0;
  HostTimer(ftm_shard_plan* p, int c) : pl(p), cat(c) {
    if (pl->hostprof) t0 = std::chrono::steady_clock::now();
  }
  ~HostTimer() {
    if (pl->hostprof)
      pl->host_ns[cat] +=
          std::chrono::duration<double, std::nano>(std::chrono::steady_clock::now() - t0).count();
  }
};
}  // namespace

namespace {

size_t elems_local(const ftm_shard_config* c) {
  const size_t R = size_t(c->shard.rows), N = size_t(c->shard.cols);
  return size_t(c->shard.batch) * kC * R * N;
}

int validate(const ftm_shard_config* c) {
  if (!c) return FTM_BAD_ARGUMENT;
  const ftm_problem& p = c->shard;
  if (c->world < 1 || c->world > FTM_MAX_RANKS || c->rank < 0 || c->rank >= c->world)
    return FTM_BAD_ARGUMENT;
  if (c->scheme != FTM_SHARD_ALLTOALL && c->scheme != FTM_SHARD_ALLGATHER) return FTM_BAD_ARGUMENT;
  if (c->scheme == FTM_SHARD_ALLGATHER && p.mode != FTM_OUTGOING) return FTM_BAD_ARGUMENT;
  if (p.c_z != kC || p.c_h != kC || p.batch < 1 || p.rows < 1) return FTM_BAD_SHAPE;
  if (p.cols != p.rows * c->world) return FTM_BAD_SHAPE;
  if (c->row_chunks < 1 || c->row_chunks > FTM_SHARD_MAX_ROW_CHUNKS) return FTM_BAD_ARGUMENT;
  if (p.batch > 1 && c->row_chunks != 1) return FTM_BAD_ARGUMENT;   // z rows are batch-strided
  if (p.rows % c->row_chunks != 0) return FTM_BAD_SHAPE;
  const int rc = p.rows / c->row_chunks;
  if (rc % 128 != 0) return FTM_BAD_SHAPE;   // row / k blocks of the contraction
  // per-destination stores of the input stage: 128 / P channels, a multiple of 16
  if (kC % c->world != 0 || (kC / c->world) % 16 != 0) return FTM_BAD_SHAPE;
  if (p.mode != FTM_OUTGOING && p.mode != FTM_INCOMING) return FTM_BAD_ARGUMENT;
  return FTM_OK;
}

int fail(cudaError_t e) { return e == cudaSuccess ? FTM_OK : FTM_LAUNCH_FAILED; }

// trace tags: (what << 8) | index
enum { T_START = 1, T_INPUT = 2, T_AB_SENT = 3, T_AB_READY = 4, T_CONTRACT = 5, T_X_SENT = 6,
       T_X_READY = 7, T_OUTPUT = 8 };
void mark(ftm_shard_plan* pl, cudaStream_t s, int what, int index) {
  if (!pl->trace || pl->trace_n >= FTM_SHARD_TRACE_POINTS) return;
  mark_kernel<<<1, 1, 0, s>>>(pl->trace, pl->trace_n++, (what << 8) | index);
}

int wait_flags(ftm_shard_plan* pl, const FlagList& fl, int kind, cudaStream_t s) {
  HostTimer ht(pl, H_WAIT);
  wait_flags_kernel<<<1, 32, 0, s>>>(pl->cfg.flags[pl->me], fl, pl->epoch, pl->cfg.err_word,
                                     (KERNEL_EXCHANGE << 8) | (kind << 4) | 1);
  ++pl->launches;
  return fail(cudaGetLastError());
}

int signal(ftm_shard_plan* pl, int q, int word) {
  HostTimer ht(pl, H_SIGNAL);
  signal_kernel<<<1, 1, 0, pl->cur>>>(pl->cfg.flags[q] + word, pl->epoch);
  ++pl->launches;
  return fail(cudaGetLastError());
}

typedef unsigned short h16;   // fp16 element, for pointer arithmetic

// Queue one run (bytes a multiple of 16) for the plan's push path: a copy-engine copy
// right away, or a run of the next push_kernel launch.
int push_run(ftm_shard_plan* pl, void* dst, const void* src, size_t bytes) {
  HostTimer ht(pl, H_COPY);
  if (!pl->sm_push) return fail(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, pl->cur));
  PushList& p = pl->pending;
  if (p.count == kMaxSegs) return FTM_BAD_ARGUMENT;
  p.src[p.count] = static_cast<const uint4*>(src);
  p.dst[p.count] = static_cast<uint4*>(dst);
  p.n16[p.count] = bytes / 16;
  ++p.count;
  return FTM_OK;
}

// Launch the queued runs (SM path) and raise `flags` of the peers in `who` (bit q) to
// the forward's epoch once they have landed; on the copy-engine path the runs are
// already queued and the flags are raised by signal kernels.
int push_flush(ftm_shard_plan* pl, unsigned who, int word) {
  int st;
  if (!pl->sm_push) {
    for (int sft = 1; sft <= pl->P; ++sft) {
      const int q = (pl->me + sft) % pl->P;
      if (who & (1u << q))
        if ((st = signal(pl, q, word)) != FTM_OK) return st;
    }
    return FTM_OK;
  }
  PushList& p = pl->pending;
  p.nflags = 0;
  for (int q = 0; q < pl->P; ++q)
    if (who & (1u << q)) p.flag[p.nflags++] = pl->cfg.flags[q] + word;
  p.epoch = pl->epoch;
  p.done = pl->push_done + (pl->cur == pl->copy ? 0 : 1);
  if (p.count || p.nflags) {
    push_kernel<<<pl->push_ctas, 256, 0, pl->cur>>>(p);
    ++pl->launches;
    if ((st = fail(cudaGetLastError())) != FTM_OK) return st;
  }
  p.count = 0;
  return FTM_OK;
}

// Owners contracted per launch: with 8 ranks one owner's block is only 128 tiles for
// 74 CTA pairs, so owners go in pairs there.
int owners_per_launch(int P) { return P >= 8 ? 2 : 1; }

int forward_alltoall(ftm_shard_plan* pl, const void* z, const float* mask, void* out,
                     cudaStream_t cs) {
  const ftm_shard_config& c = pl->cfg;
  const int P = pl->P, me = pl->me, RC = pl->RC, rc = pl->rc, R = pl->R, N = pl->N, B = pl->B;
  const int lq = pl->lq;
  const bool incoming = c.shard.mode == FTM_INCOMING;
  const size_t unit = pl->unit;                                  // rc * N
  const size_t blk = size_t(B) * lq * unit;                      // a (or b) of one (dest, chunk)
  const size_t slot_elems = 2 * elems_local(&c);                 // a and b of one receive slot
  const int slot = pl->epoch & 1;
  int st;
  // Local layout, chunk-major: [chunk r][dest q][a | b][batch][lq][rc][N] (incoming: the
  // transposed [lq][N][rc] planes), written by the input stage's per-destination stores,
  // so the a and b pieces rank q needs from chunk r are one contiguous run.
  if ((st = fail(cudaStreamWaitEvent(cs, pl->ev_pushed, 0))) != FTM_OK) return st;
  mark(pl, cs, T_START, 0);
  for (int r = 0; r < RC; ++r) {
    ftm_problem sub = c.shard;
    sub.rows = rc;
    h16* chunk = static_cast<h16*>(c.a_local) + size_t(r) * P * 2 * blk;
    ftm_peer_planes pa{}, pb{};
    pa.world = pb.world = P;
    pa.rank = pb.rank = 0;
    for (int q = 0; q < P; ++q) {
      pa.base[q] = chunk + size_t(q) * 2 * blk;
      pb.base[q] = chunk + size_t(q) * 2 * blk + blk;
    }
    const h16* z_r = static_cast<const h16*>(z) + size_t(r) * rc * N * kC;
    const float* m_r = mask ? mask + size_t(r) * rc * N : nullptr;
    HostTimer ht(pl, H_INPUT);
    if ((st = ftm_input_stage_scatter(&sub, z_r, m_r, c.packed, &pa, &pb,
                                      c.zstats + size_t(r) * rc * N * 2, c.err_word, cs)) != FTM_OK)
      return st;
    ++pl->launches;
    mark(pl, cs, T_INPUT, r);
    if ((st = fail(cudaEventRecord(pl->ev_in[r], cs))) != FTM_OK) return st;
    if ((st = fail(cudaStreamWaitEvent(pl->copy, pl->ev_in[r], 0))) != FTM_OK) return st;
    // shifted order: at any moment every rank sends to a different peer; own piece last
    for (int sft = 1; sft <= P; ++sft) {
      const int q = (me + sft) % P;
      h16* dst = static_cast<h16*>(c.recv_a[q]) + size_t(slot) * slot_elems +
                 size_t(me * RC + r) * 2 * blk;
      if ((st = push_run(pl, dst, chunk + size_t(q) * 2 * blk, 2 * blk * 2)) != FTM_OK) return st;
      if (!pl->sm_push) mark(pl, pl->copy, T_AB_SENT, q * 16 + r);
    }
    // receivers need every chunk before they contract: one flag per peer, raised after
    // the last chunk
    if ((st = push_flush(pl, r == RC - 1 ? (1u << P) - 1 : 0u, kFlagAB + me)) != FTM_OK) return st;
    if (pl->sm_push) mark(pl, pl->copy, T_AB_SENT, r);
  }
  if ((st = fail(cudaEventRecord(pl->ev_pushed, pl->copy))) != FTM_OK) return st;

  FlagList fl{};
  for (int s = 0; s < P; ++s) fl.idx[fl.count++] = kFlagAB + s;
  if ((st = wait_flags(pl, fl, 1, cs)) != FTM_OK) return st;
  mark(pl, cs, T_AB_READY, 0);
  // the previous forward's x pushes must be done reading the x blocks
  if ((st = fail(cudaStreamWaitEvent(cs, pl->ev_x_pushed, 0))) != FTM_OK) return st;

  pl->cur = pl->copy_x;
  // received: [slot][src s][chunk r][a | b][batch][lq][rc][N]
  const h16* Rs = static_cast<const h16*>(c.recv_a[me]) + size_t(slot) * slot_elems;
  const size_t owner_elems = size_t(B) * lq * R * N;
  const int G = owners_per_launch(P), groups = P / G, my_group = me / G;
  const bool direct_own = (G == 1 && B == 1);
  for (int gs = 1; gs <= groups; ++gs) {
    const int g = (my_group + gs) % groups, o0 = g * G;
    ftm_contraction_layout d{};
    d.L = B * lq; d.m = G * R; d.n = N; d.k = N;
    if (!incoming) {
      // row blocks (src, chunk) of rc rows; owners o0.. have blocks [o0*RC, (o0+G)*RC)
      d.k_per_block = N;
      d.a = Rs + size_t(o0) * RC * 2 * blk; d.a_rows_per_block = rc;
      d.a_block_stride = 2 * blk; d.a_l_stride = unit; d.a_row_stride = N;
      d.b = Rs + blk; d.b_rows_per_block = rc;
      d.b_block_stride = 2 * blk; d.b_l_stride = unit; d.b_row_stride = N;
    } else {
      // k blocks (src, chunk) of rc; planes [l][i][k in block]; owners' rows i
      d.k_per_block = rc;
      d.a = Rs + size_t(o0) * R * rc; d.a_rows_per_block = G * R;
      d.a_l_stride = unit; d.a_row_stride = rc; d.a_kblock_stride = 2 * blk;
      d.b = Rs + blk; d.b_rows_per_block = N;
      d.b_l_stride = unit; d.b_row_stride = rc; d.b_kblock_stride = 2 * blk;
    }
    const bool direct = direct_own && o0 == me;
    d.x = direct ? static_cast<void*>(static_cast<h16*>(c.x_plane[me]) + size_t(me) * lq * R * N)
                 : static_cast<void*>(static_cast<h16*>(c.x_blocks) + size_t(o0) * owner_elems);
    d.x_rows_per_block = R; d.x_block_stride = owner_elems; d.x_l_stride = size_t(R) * N;
    d.x_row_stride = N;
    {
      HostTimer ht(pl, H_CONTRACT);
      if ((st = ftm_contraction_general(&d, c.err_word, cs)) != FTM_OK) return st;
    }
    ++pl->launches;
    mark(pl, cs, T_CONTRACT, g);
    if (direct) continue;
    if ((st = fail(cudaEventRecord(pl->ev_owner[g], cs))) != FTM_OK) return st;
    if ((st = fail(cudaStreamWaitEvent(pl->copy_x, pl->ev_owner[g], 0))) != FTM_OK) return st;
    for (int o = o0; o < o0 + G; ++o) {
      const h16* src = static_cast<const h16*>(c.x_blocks) + size_t(o) * owner_elems;
      h16* dst = static_cast<h16*>(c.x_plane[o]) + size_t(me) * lq * R * N;
      // own block: a local copy on the same stream, ahead of this rank's wait for x
      for (int b = 0; b < B; ++b)
        if ((st = push_run(pl, dst + size_t(b) * kC * R * N, src + size_t(b) * lq * R * N,
                           size_t(lq) * R * N * 2)) != FTM_OK)
          return st;
      if (!pl->sm_push) mark(pl, pl->copy_x, T_X_SENT, o);
    }
    if (pl->sm_push) {
      if ((st = push_flush(pl, 0u, 0)) != FTM_OK) return st;
      mark(pl, pl->copy_x, T_X_SENT, g);
    }
  }
  // owners wait for every source's x: one flag per owner, after the last push
  unsigned who = 0;
  for (int o = 0; o < P; ++o)
    if (!(o == me && direct_own)) who |= 1u << o;
  if ((st = push_flush(pl, who, kFlagX + me)) != FTM_OK) return st;
  if ((st = fail(cudaEventRecord(pl->ev_x_pushed, pl->copy_x))) != FTM_OK) return st;
  FlagList fx{};
  for (int s = 0; s < P; ++s)
    if (s != me || !direct_own) fx.idx[fx.count++] = kFlagX + s;
  if (fx.count && (st = wait_flags(pl, fx, 2, cs)) != FTM_OK) return st;
  mark(pl, cs, T_X_READY, 0);
  ++pl->launches;
  HostTimer ht(pl, H_OUTPUT);
  st = ftm_output_stage(&pl->out_problem, z, mask, c.x_plane[me], c.zstats, c.packed, out,
                        c.err_word, cs);
  mark(pl, cs, T_OUTPUT, 0);
  return st;
}

int forward_allgather(ftm_shard_plan* pl, const void* z, const float* mask, void* out,
                      cudaStream_t cs) {
  const ftm_shard_config& c = pl->cfg;
  const int P = pl->P, me = pl->me, RC = pl->RC, rc = pl->rc, R = pl->R, N = pl->N;
  const int L = pl->L;
  const size_t unit = pl->unit;
  const size_t blk = size_t(L) * unit;                     // one (src, chunk) block of b
  const size_t slot_elems = size_t(P) * RC * blk;
  const int slot = pl->epoch & 1;
  int st;
  h16* own = static_cast<h16*>(c.recv_b[me]) + size_t(slot) * slot_elems;
  if ((st = fail(cudaStreamWaitEvent(cs, pl->ev_pushed, 0))) != FTM_OK) return st;
  mark(pl, cs, T_START, 0);
  for (int r = 0; r < RC; ++r) {
    ftm_problem sub = c.shard;
    sub.rows = rc;
    h16* a_r = static_cast<h16*>(c.a_local) + size_t(r) * blk;
    h16* b_r = own + size_t(me * RC + r) * blk;             // b goes straight to its block
    const h16* z_r = static_cast<const h16*>(z) + size_t(r) * rc * N * kC;
    const float* m_r = mask ? mask + size_t(r) * rc * N : nullptr;
    if ((st = ftm_input_stage(&sub, z_r, m_r, c.packed, a_r, b_r, c.zstats + size_t(r) * rc * N * 2,
                              c.err_word, cs)) != FTM_OK)
      return st;
    ++pl->launches;
    mark(pl, cs, T_INPUT, r);
    if ((st = fail(cudaEventRecord(pl->ev_in[r], cs))) != FTM_OK) return st;
    if ((st = fail(cudaStreamWaitEvent(pl->copy, pl->ev_in[r], 0))) != FTM_OK) return st;
    for (int sft = 1; sft < P; ++sft) {
      const int q = (me + sft) % P;
      h16* dst = static_cast<h16*>(c.recv_b[q]) + size_t(slot) * slot_elems + size_t(me * RC + r) * blk;
      if ((st = push_run(pl, dst, b_r, blk * 2)) != FTM_OK) return st;
      if ((st = push_flush(pl, 1u << q, kFlagAB + me * FTM_SHARD_MAX_ROW_CHUNKS + r)) != FTM_OK)
        return st;
      mark(pl, pl->copy, T_AB_SENT, q * 16 + r);
    }
  }
  if ((st = fail(cudaEventRecord(pl->ev_pushed, pl->copy))) != FTM_OK) return st;
  // columns of source s, chunk r: B = that block (rc rows), X columns [s R + r rc, + rc)
  auto contract = [&](int s, int r0, int nr) -> int {
    ftm_contraction_layout d{};
    d.L = L; d.m = R; d.n = nr * rc; d.k = N; d.k_per_block = N;
    d.a = c.a_local; d.a_rows_per_block = rc;
    d.a_block_stride = blk; d.a_l_stride = unit; d.a_row_stride = N;
    d.b = own + size_t(s * RC + r0) * blk; d.b_rows_per_block = rc;
    d.b_block_stride = blk; d.b_l_stride = unit; d.b_row_stride = N;
    d.x = static_cast<h16*>(c.x_blocks) + size_t(s) * R + size_t(r0) * rc;
    d.x_rows_per_block = R; d.x_l_stride = size_t(R) * N; d.x_row_stride = N;
    ++pl->launches;
    return ftm_contraction_general(&d, c.err_word, cs);
  };
  if ((st = contract(me, 0, RC)) != FTM_OK) return st;      // own b: no wait
  mark(pl, cs, T_CONTRACT, me * 16);
  for (int sft = 1; sft < P; ++sft) {
    const int s = (me + P - sft) % P;                          // the order peers send to us
    for (int r = 0; r < RC; ++r) {
      FlagList fl{};
      fl.idx[fl.count++] = kFlagAB + s * FTM_SHARD_MAX_ROW_CHUNKS + r;
      if ((st = wait_flags(pl, fl, 1, cs)) != FTM_OK) return st;
      mark(pl, cs, T_AB_READY, s * 16 + r);
      if ((st = contract(s, r, 1)) != FTM_OK) return st;
      mark(pl, cs, T_CONTRACT, s * 16 + r);
    }
  }
  ++pl->launches;
  st = ftm_output_stage(&pl->out_problem, z, mask, c.x_blocks, c.zstats, c.packed, out,
                        c.err_word, cs);
  mark(pl, cs, T_OUTPUT, 0);
  return st;
}

}  // namespace

extern "C" {

size_t ftm_shard_buffer_bytes(const ftm_shard_config* cfg, int which) {
  if (validate(cfg) != FTM_OK) return 0;
  const size_t local = elems_local(cfg) * 2;
  const size_t R = size_t(cfg->shard.rows), N = size_t(cfg->shard.cols), B = size_t(cfg->shard.batch);
  switch (which) {
    case FTM_SHARD_BUF_LOCAL:
      return cfg->scheme == FTM_SHARD_ALLTOALL ? 2 * local : local;
    case FTM_SHARD_BUF_ZSTATS: return B * R * N * 8;
    case FTM_SHARD_BUF_XBLOCKS: return local;
    case FTM_SHARD_BUF_RECV:   // two slots; alltoall: a and b, allgather: b of every rank
      return cfg->scheme == FTM_SHARD_ALLGATHER ? 2 * local * size_t(cfg->world) : 4 * local;
    case FTM_SHARD_BUF_XPLANE: return local;
    case FTM_SHARD_BUF_FLAGS: return FTM_SHARD_FLAG_WORDS * sizeof(int);
    default: return 0;
  }
}

int ftm_shard_plan_create(const ftm_shard_config* cfg, ftm_shard_plan** plan) {
  if (!plan) return FTM_BAD_ARGUMENT;
  *plan = nullptr;
  int st = validate(cfg);
  if (st != FTM_OK) return st;
  const bool a2a = cfg->scheme == FTM_SHARD_ALLTOALL;
  if (!cfg->packed || !cfg->a_local || !cfg->zstats || !cfg->x_blocks || !cfg->err_word)
    return FTM_BAD_ARGUMENT;
  for (int q = 0; q < cfg->world; ++q) {
    if (!cfg->flags[q]) return FTM_BAD_ARGUMENT;
    if (a2a && (!cfg->recv_a[q] || !cfg->x_plane[q])) return FTM_BAD_ARGUMENT;
    if (!a2a && !cfg->recv_b[q]) return FTM_BAD_ARGUMENT;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || ftm_device_supported(dev) != 1)
    return FTM_UNSUPPORTED_ARCH;
  ftm_shard_plan* pl = new (std::nothrow) ftm_shard_plan();
  if (!pl) return FTM_LAUNCH_FAILED;
  pl->cfg = *cfg;
  pl->P = cfg->world;
  pl->me = cfg->rank;
  pl->RC = cfg->row_chunks;
  pl->R = cfg->shard.rows;
  pl->N = cfg->shard.cols;
  pl->B = cfg->shard.batch;
  pl->rc = pl->R / pl->RC;
  pl->L = pl->B * kC;
  pl->lq = kC / pl->P;
  pl->unit = size_t(pl->rc) * pl->N;
  pl->dev = dev;
  pl->epoch = 0;
  // FTM_SHARD_PUSH=sm: pushes by a kernel of FTM_SHARD_PUSH_CTAS CTAs (default 32) doing
  // vector stores into the peers' windows, instead of copy-engine copies
  {
    const char* v = getenv("FTM_SHARD_PUSH");
    pl->sm_push = (v && strcmp(v, "sm") == 0) ? 1 : 0;
    const char* n = getenv("FTM_SHARD_PUSH_CTAS");
    pl->push_ctas = n ? atoi(n) : 32;
    if (pl->push_ctas < 1) pl->push_ctas = 1;
    if (pl->push_ctas > 1024) pl->push_ctas = 1024;
    // the counter lives in the last word of this rank's flag buffer (zeroed by the caller,
    // never written by peers)
    pl->push_done = reinterpret_cast<unsigned int*>(cfg->flags[cfg->rank] + FTM_SHARD_FLAG_WORDS - 2);
  }
  {
    const char* hp = getenv("FTM_SHARD_HOSTPROF");
    pl->hostprof = (hp && strcmp(hp, "1") == 0) ? 1 : 0;
  }
  bool ok = cudaStreamCreateWithFlags(&pl->copy, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&pl->copy_x, cudaStreamNonBlocking) == cudaSuccess;
  for (int i = 0; ok && i < FTM_SHARD_MAX_ROW_CHUNKS; ++i)
    ok = cudaEventCreateWithFlags(&pl->ev_in[i], cudaEventDisableTiming) == cudaSuccess;
  for (int i = 0; ok && i < FTM_MAX_RANKS; ++i)
    ok = cudaEventCreateWithFlags(&pl->ev_owner[i], cudaEventDisableTiming) == cudaSuccess;
  ok = ok && cudaEventCreateWithFlags(&pl->ev_pushed, cudaEventDisableTiming) == cudaSuccess;
  ok = ok && cudaEventCreateWithFlags(&pl->ev_x_pushed, cudaEventDisableTiming) == cudaSuccess;
  // recorded once so the first forward's waits on them are satisfied
  ok = ok && cudaEventRecord(pl->ev_pushed, pl->copy) == cudaSuccess;
  ok = ok && cudaEventRecord(pl->ev_x_pushed, pl->copy_x) == cudaSuccess;
  if (!ok) {
    ftm_shard_plan_destroy(pl);
    return FTM_LAUNCH_FAILED;
  }
  *plan = pl;
  return FTM_OK;
}

int ftm_shard_forward(ftm_shard_plan* plan, const void* z, const float* mask, void* out,
                      int32_t out_dtype, ftm_stream_t stream) {
  set_last_launch_count(0);
  if (!plan || !z || !out) return FTM_BAD_ARGUMENT;
  if (out_dtype != FTM_F16 && out_dtype != FTM_BF16 && out_dtype != FTM_F32) return FTM_BAD_DTYPE;
  plan->out_problem = plan->cfg.shard;
  plan->out_problem.out_dtype = out_dtype;
  if ((reinterpret_cast<uintptr_t>(z) & 15u) || (reinterpret_cast<uintptr_t>(out) & 15u) ||
      (reinterpret_cast<uintptr_t>(mask) & 15u))
    return FTM_BAD_ALIGN;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != plan->dev) return FTM_BAD_ARGUMENT;
  ++plan->epoch;
  plan->launches = 0;
  plan->trace_n = 0;
  plan->cur = plan->copy;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  int st;
  {
    HostTimer ht(plan, H_TOTAL);
    st = plan->cfg.scheme == FTM_SHARD_ALLTOALL ? forward_alltoall(plan, z, mask, out, cs)
                                                : forward_allgather(plan, z, mask, out, cs);
  }
  ++plan->forwards;
  // the stage entry points set the per-thread count to 1 each; report the forward's total
  set_last_launch_count(st == FTM_OK ? plan->launches : 0);
  return st;
}

int ftm_shard_set_trace(ftm_shard_plan* plan, long long* trace) {
  if (!plan) return FTM_BAD_ARGUMENT;
  plan->trace = trace;
  return FTM_OK;
}

void ftm_shard_plan_destroy(ftm_shard_plan* plan) {
  if (!plan) return;
  if (plan->hostprof && plan->forwards) {
    fprintf(stderr, "ftm_shard rank %d: host us per forward over %lld forwards:", plan->me,
            plan->forwards);
    for (int i = 0; i < H_COUNT; ++i)
      fprintf(stderr, " %s %.1f;", kHostNames[i], plan->host_ns[i] / 1e3 / plan->forwards);
    fprintf(stderr, "\n");
  }
  if (plan->copy) cudaStreamSynchronize(plan->copy);
  if (plan->copy_x) cudaStreamSynchronize(plan->copy_x);
  for (int i = 0; i < FTM_SHARD_MAX_ROW_CHUNKS; ++i)
    if (plan->ev_in[i]) cudaEventDestroy(plan->ev_in[i]);
  for (int i = 0; i < FTM_MAX_RANKS; ++i)
    if (plan->ev_owner[i]) cudaEventDestroy(plan->ev_owner[i]);
  if (plan->ev_pushed) cudaEventDestroy(plan->ev_pushed);
  if (plan->ev_x_pushed) cudaEventDestroy(plan->ev_x_pushed);
  if (plan->copy) cudaStreamDestroy(plan->copy);
  if (plan->copy_x) cudaStreamDestroy(plan->copy_x);
  delete plan;
}

}  // extern "C"
