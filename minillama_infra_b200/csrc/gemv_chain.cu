// gemv_chain.cu -- a decode step's chain of batch-1 INT8 group-64 GEMVs in one
// persistent launch (sm_100a).
//
// A Llama decode step is a chain of small GEMVs (per layer: q, k, v, o, gate,
// up, down) whose activations depend on one another: o reads the attention
// output of q/k/v, gate/up the normalised residual after o, down the SwiGLU of
// gate/up, the next layer's q/k/v the normalised residual after down.
// Launched one by one, every GEMV pays a kernel boundary (the previous grid
// drains, the next one fills its pipeline), and a 1-4 MB GEMV streams for well
// under a microsecond, so the boundaries, not HBM, set the step time.
//
// Here one CTA per SM streams the weights of the whole chain without a
// kernel boundary:
//
//  * Work units.  Every GEMV is cut into stages of whole rows (64 row slices
//    of 1024 columns for W8A32, 32 of 2048 for W8A8: 64 KB of weights plus
//    their scales), the stages of all GEMVs are numbered in chain order, and
//    each run of ops that adds no new dependency (a "phase") is spread over
//    all CTAs.  Each CTA moves its units through a ring of shared-memory
//    slots with 1-D bulk copies; weights never depend on an activation, so the
//    ring runs ahead across GEMV boundaries and across dependency waits.
//  * Dependencies travel with the data.  Every op writes each finished row
//    twice: into its y, and into the chain's mirror of that op as one 8-byte
//    word {value, tag}, tag = (launch sequence << 16) | op index, with a
//    single relaxed 64-bit store (single-copy atomic: a reader sees the value
//    and its tag together, and no fence is needed).  An op whose activation
//    is an earlier op's output reads that op's mirror and retries every word
//    until it carries the producer's tag: readiness and data arrive in the
//    same L2 load.  An op waits for ops [0, wait) of the chain; the ones not
//    implied by its activation's producer (whose rows were written only after
//    ITS wait was met) are checked the same way, by their mirrors' tags (o
//    waits for k and v, for instance).  Every wait is bounded in time and
//    records a device error instead of hanging.
//  * Activations.  When the activation changes the consumers load it
//    (tag-checked, or plainly for an input that is ready at launch) and
//    prepare it: an optional RMSNorm (weight * (x / sqrt(mean(x^2) + 1e-5)),
//    the reference's rmsnorm_cuda / fused_add_rmsnorm_cuda before the q/k/v
//    and gate/up projections, recomputed by every CTA from the whole vector),
//    then W8A32 digit-pair planes (digit_quad) or the fused W8A8 quantisation
//    (quant_quad) -- once per CTA into shared memory, or, when every warp owns
//    its own slice of the row (W8A32 with n = 8192, no norm), by each warp in
//    registers without a barrier.
//  * Warp roles: consumer warps compute rows from the ring, and the last one
//    to finish with a slot stores its rows and frees the slot; one producer
//    warp refills freed slots (issuing a bulk copy takes long enough that it
//    is kept off the consumers).
//  * Rows are computed exactly as in gemv_stream_kernel (same row kernels,
//    same slice order), so an op without a norm prologue gives bit-identical
//    output to the corresponding mli_gemv_* call.
//  * Row-sharded chains (one process per GPU): an op computes a row range of a
//    larger GEMV and stores each row, tagged, into every rank's mirror over
//    NVLink (plain system-scope peer stores); a reader of the whole vector
//    checks the tags of words other GPUs wrote.  Mirrors are kept twice,
//    alternating by launch, so a rank one launch ahead never overwrites words
//    another is still reading.
//  * A chain in which no op reads another's rows runs a kernel compiled
//    without any of the mirror, tag, poll or peer code.
//  * Every CTA processes its units in chain order and a unit only waits for
//    earlier ops, so the earliest unfinished op never waits: with all CTAs
//    resident (cooperative launch) the chain cannot deadlock.  The last CTA to
//    finish advances the launch sequence, so the next launch (or graph
//    replay) needs no host-side reset and never takes an old row for a new
//    one.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>

// Built as a device module of its own (no -rdc): ptxas then sizes the
// out-of-line prologues within the kernel's register budget.  The library's
// device error word is reached through a pointer (Args::err).
#define MLI_SEPARATE_DEVICE_MODULE
#include "gemv_rows.cuh"
#include "mli_common.cuh"
#include "mli_internal.h"

namespace mli {
namespace chain {

constexpr int kMaxRing = 6;
constexpr int kHeader = 256;
constexpr int kMaxSlices = 8;
constexpr int kMaxOps = 1 << 16;
// The launch sequence runs 1 .. 65534: an even period, so consecutive launches
// always alternate between the two halves of a sharded chain's mirrors.
constexpr unsigned kSeqPeriod = 65534;
constexpr int kMaxPeers = 8;  // ranks of a sharded chain

// Row epilogues: store y = v; add into y (the residual adds after the
// reference's o and down projections, src/model_cuda_v2_shared.cu:99-118,
// :215-218, :414); SwiGLU with the next op (gate = this op, up = the next one,
// stored as (g * (1 / (1 + expf(-g)))) * u, :220-227, :410); the companion up
// op of a SwiGLU pair (no units of its own).
constexpr int kEpiStore = 0, kEpiAdd = 1, kEpiSwiglu = 2, kEpiCompanion = 3;

// Device-side descriptor of one GEMV of the chain, 112 bytes (geometry
// precomputed on the host, as plan_stream does for the single-GEMV kernel).
// Kernels copy the table into shared memory when it fits.
struct Op {
  float* y;
  const void* act;       // fp32 x (W8A32, fused W8A8) or int8 xq (W8A8)
  const float* xs;       // W8A8 activation scale
  const int8_t* w;
  const float* s;
  const float* norm_w;   // RMSNorm weights of the activation (nullptr: none)
  int n, d;              // in / out features
  int unit_base;         // first work unit of this op
  int wait;              // ops [0, wait) complete before this op reads its activation
  int epoch;             // ops of one epoch read the same prepared activation
  int src;               // op whose mirror holds the activation (-1: `act`, ready at launch)
  int base;              // ADD: op whose mirror holds y before this op (-1: y itself)
  int mirror;            // word offset of this op's mirror (-1: none)
  int poll_first;        // other ops of the wait prefix to check: polls[poll_first, +poll_count)
  int poll_count;
  uint8_t S;             // slices per row
  uint8_t epi;           // kEpi*: how a finished row is stored
  uint16_t R;            // rows per stage (a SwiGLU stage: R/2 gate rows, then the R/2 up rows)
  int row_off;           // row of the whole (row-sharded) GEMV this op's row 0 is
  int d_total;           // rows of the whole GEMV: the length of this op's mirror
  int pad[3];
  __host__ __device__ const float* x() const { return static_cast<const float*>(act); }
  // output rows per work unit
  __host__ __device__ int Ru() const { return epi == kEpiSwiglu ? R / 2 : R; }
  __host__ __device__ const int8_t* xq() const { return static_cast<const int8_t*>(act); }
  __host__ __device__ int G() const { return n / kGroup; }
};
static_assert(sizeof(Op) == 112 && sizeof(Op) % 16 == 0, "chain op descriptor: 112 bytes, copied as uint4s");

struct Args {
  const Op* ops;        // global copy of the table
  const int* phases;    // [n_phases + 1] first unit of every phase, then the unit count
  const int* polls;     // [n_polls] op indices checked by tag (see Op::poll_first)
  uint32_t table_off;   // shared-memory copy of ops, phases, polls (0: read them from global)
  int n_phases;
  int count;
  int n_polls;
  int units;            // stages of all ops
  uint64_t* mirror;     // every op's rows as {value, tag} words (this rank's block)
  uint64_t* const* peers;  // sharded chains: every rank's mirror block (the own one included)
  int world;            // ranks of a sharded chain (1: rows stay on this GPU)
  uint32_t mirror_half; // words from a mirror to its copy for odd launches (0: one copy)
  unsigned* seq;        // launch sequence, 1 .. kSeqPeriod (advanced by the last CTA)
  unsigned* finished;   // CTAs finished in this launch
  int ring;
  uint32_t slot_bytes;  // ring slot: the largest stage of the chain
  uint32_t x_off, ring_off, part_off;
  int part_stride;      // floats of split-K partials per slot
  unsigned* err;        // the library's device error word (first code wins)
};

__device__ __forceinline__ void record_error(const Args& a, unsigned code) {
  if (a.err) atomicCAS(a.err, 0u, code);
}

// Shared-memory header: full[6] @0, free[6] @48, per-slot warp counters @96,
// flags @128..140, the launch sequence @140, two reduction arrays of one
// float per consumer warp @160 (quantiser) and @208 (RMSNorm).
struct Smem {
  uint64_t* full;   // weights of the slot's unit landed (bulk copy)
  uint64_t* free;   // the consumers are done with the slot: it may be refilled
  int* counters;
  volatile int* broken;
  int* issued;
  int* last_cta;
  unsigned* seq;
  float* red;
  float* red2;
  __device__ explicit Smem(unsigned char* b)
      : full(reinterpret_cast<uint64_t*>(b)),
        free(reinterpret_cast<uint64_t*>(b + 48)),
        counters(reinterpret_cast<int*>(b + 96)),
        broken(reinterpret_cast<volatile int*>(b + 128)),
        issued(reinterpret_cast<int*>(b + 132)),
        last_cta(reinterpret_cast<int*>(b + 136)),
        seq(reinterpret_cast<unsigned*>(b + 140)),
        red(reinterpret_cast<float*>(b + 160)),
        red2(reinterpret_cast<float*>(b + 208)) {}
};
static_assert(208 + 12 * 4 <= kHeader, "shared-memory header");

__host__ __device__ __forceinline__ uint32_t row_tag(unsigned seq, int op) {
  return (seq << 16) | static_cast<uint32_t>(op & 0xffff);
}

// Mirror words are read with GPU-scope relaxed loads, or system-scope ones
// when other GPUs write them (a sharded chain).
__device__ __forceinline__ void ld_relaxed_v2(const uint64_t* p, uint64_t& a, uint64_t& b, bool sys) {
  if (sys)
    asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
  else
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_b64(const uint64_t* p, bool sys) {
  uint64_t v;
  if (sys)
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  else
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_b64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t tagged(float v, uint32_t tag) {
  return (static_cast<uint64_t>(tag) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ bool has_tag(uint64_t w, uint32_t tag) {
  return static_cast<uint32_t>(w >> 32) == tag;
}
__device__ __forceinline__ float word_value(uint64_t w) {
  return __uint_as_float(static_cast<uint32_t>(w));
}

// Four consecutive tagged words already loaded: their values when all four
// carry `tag`; otherwise they are reloaded (16-byte aligned p) until they do,
// false once `kWaitLimitNs` have passed since t0.
__device__ __forceinline__ bool all_tagged4(uint64_t w0, uint64_t w1, uint64_t w2, uint64_t w3, uint32_t tag) {
  return has_tag(w0, tag) && has_tag(w1, tag) && has_tag(w2, tag) && has_tag(w3, tag);
}
// Spinning readers back off between polls, so that thousands of threads
// waiting for the same few kilobytes do not crowd the L2 slices their
// producers are writing to.
__device__ __forceinline__ void poll_backoff(unsigned& ns) {
  __nanosleep(ns);
  ns = ns < 256 ? 2 * ns : 256;
}
// Op holding global unit u, searching forward from op `o` (units grow).
__device__ __forceinline__ int find_op(const Op* ops, int count, int u, int o) {
  while (o + 1 < count && ops[o + 1].unit_base <= u) ++o;
  return o;
}

// A CTA's units, in chain order: in every phase (a run of ops that needs no
// new dependency), CTA c of G takes the contiguous range
// [start + c T / G, start + (c + 1) T / G) of the phase's T units.  Without
// dependencies a CTA thus touches only a few ops (few activation changes);
// with them every phase is still spread over all SMs.
struct Cursor {
  const int* ph;
  int n_ph, cta, grid;
  int p, u, hi;
  __device__ void range() {
    for (; p < n_ph; ++p) {
      const long long lo = ph[p], t = ph[p + 1] - ph[p];
      u = static_cast<int>(lo + t * cta / grid);
      hi = static_cast<int>(lo + t * (cta + 1) / grid);
      if (u < hi) return;
    }
    u = hi = 0;
  }
  __device__ Cursor(const int* phases, int n, int c, int g) : ph(phases), n_ph(n), cta(c), grid(g), p(0) {
    range();
  }
  __device__ bool valid() const { return p < n_ph; }
  __device__ void next() {
    if (++u >= hi) {
      ++p;
      range();
    }
  }
};

// Units of CTA `cta` in all phases.
__device__ __forceinline__ int cta_units(const int* ph, int n_ph, int cta, int grid) {
  int c = 0;
  for (int p = 0; p < n_ph; ++p) {
    const long long lo = ph[p], t = ph[p + 1] - ph[p];
    c += static_cast<int>(lo + t * (cta + 1) / grid - (lo + t * cta / grid));
  }
  return c;
}

// Bulk copies of unit u (a stage of op o) into ring slot `slot`.
template <bool kEpi>
__device__ __forceinline__ void issue_unit(const Args& a, const Op* ops, unsigned char* ring,
                                           uint64_t* full, int o, int u, int slot) {
  const Op& op = ops[o];
  const int R = op.R, G = op.G(), Ru = kEpi ? op.Ru() : R;
  const int row0 = (u - op.unit_base) * Ru;
  const int rows = min(Ru, op.d - row0);
  const uint32_t wb = static_cast<uint32_t>(rows) * op.n;
  const uint32_t sb = static_cast<uint32_t>(rows) * G * 4u;
  unsigned char* dst = ring + static_cast<size_t>(slot) * a.slot_bytes;
  const bool glu = kEpi && op.epi == kEpiSwiglu;
  mbar_arrive_expect_tx(&full[slot], glu ? 2 * (wb + sb) : wb + sb);
  bulk_copy_g2s(dst, op.w + static_cast<size_t>(row0) * op.n, wb, &full[slot]);
  bulk_copy_g2s(dst + static_cast<size_t>(R) * op.n, op.s + static_cast<size_t>(row0) * G, sb,
                &full[slot]);
  if (glu) {  // the up projection's same rows behind the gate's
    const Op& up = ops[o + 1];
    bulk_copy_g2s(dst + static_cast<size_t>(Ru) * op.n, up.w + static_cast<size_t>(row0) * op.n, wb,
                  &full[slot]);
    bulk_copy_g2s(dst + static_cast<size_t>(R) * op.n + static_cast<size_t>(Ru) * G * 4u,
                  up.s + static_cast<size_t>(row0) * G, sb, &full[slot]);
  }
}

// Offset of this launch's copy of the mirrors (sharded chains keep two,
// alternating by launch, so that a rank already in the next launch never
// overwrites words another rank is still reading).
__device__ __forceinline__ uint32_t mirror_half(const Args& a, unsigned seq) { return (seq & 1u) ? a.mirror_half : 0u; }

// Consumer threads check, by their mirrors' tags, that every row of the ops
// polls[first, first + count) was written in this launch.  The polled ops'
// rows form one index space; a thread's words of one pass (up to 8) are all in
// flight before the first is checked.  False if a row did not arrive in time.
template <int kT>
__device__ __forceinline__ bool poll_ops(const Args& a, const Op* ops, const int* polls, int first, int count,
                                         unsigned seq) {
  const uint64_t t0 = global_timer_ns();
  const bool sys = a.world > 1;
  const uint32_t half = mirror_half(a, seq);
  int total = 0;
  for (int p = first; p < first + count; ++p) total += ops[polls[p]].d_total;
  int p = first, start = 0;  // op polls[p] holds rows [start, start + d_total) of the space
  for (int r0 = threadIdx.x; r0 < total; r0 += 8 * kT) {
    const uint64_t* addr[8];
    uint32_t tags[8];
    unsigned pending = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = r0 + k * kT;
      addr[k] = a.mirror;
      tags[k] = 0;
      if (i < total) {
        while (i >= start + ops[polls[p]].d_total) start += ops[polls[p++]].d_total;
        const int j = polls[p];
        addr[k] = a.mirror + half + ops[j].mirror + (i - start);
        tags[k] = row_tag(seq, j);
        pending |= 1u << k;
      }
    }
    unsigned ns = 32;
    while (true) {
      uint64_t w[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) w[k] = ((pending >> k) & 1u) ? ld_relaxed_b64(addr[k], sys) : 0ull;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (((pending >> k) & 1u) && has_tag(w[k], tags[k])) pending &= ~(1u << k);
      if (pending == 0) break;
      if (global_timer_ns() - t0 > kWaitLimitNs) return false;
      poll_backoff(ns);
    }
  }
  return true;
}

// Polls of the wait prefix, run by the activation loaders while their own
// loads are in flight (nothing to poll: always true).
struct NoPoll {
  __device__ bool operator()() const { return true; }
};
template <int kT>
struct PrefixPoll {
  const Args& a;
  const Op* ops;
  const int* polls;
  int first, count;
  unsigned seq;
  bool on;
  __device__ bool operator()() const { return !on || poll_ops<kT>(a, ops, polls, first, count, seq); }
};

// ---------------------------------------------------------------------------
// Activation preparation.  A produced activation is read from its producer's
// mirror with tag checks, one that is ready at launch with L2 loads; every
// load of a thread is in flight before the first is used.
// ---------------------------------------------------------------------------
constexpr int kPre = 8;  // float4 of activation held per consumer thread

// Float4 groups of tagged words (4 words each) a thread has in flight before it
// checks the first: kBatch, or all kPre where the kernel's registers allow
// (the shared preparation of the fused W8A8 kernels, the per-warp preparation
// of the W8A32 kernels with 8 rows per warp).
constexpr int kBatch = 4;

// Loads groups [b, b + kB) of a thread's float4 groups of tagged words into
// v, every load of the batch in flight before the first is checked, then
// reloads the words without the tag until they carry it.  `addr(j)` is the
// first word of group j (nullptr: outside the activation, v[j] = 0).
// `between` runs once the batch's loads are issued (the wait prefix's polls).
// False on a timeout or when `between` fails.
template <int kB, int J, class Addr, class Between>
__device__ __forceinline__ bool load_tagged_batch(int b, const Addr& addr, uint32_t tag, bool sys, uint64_t t0,
                                                  float4 (&v)[J], const Between& between) {
  uint64_t w[kB][4];
  unsigned pending = 0;
#pragma unroll
  for (int j = 0; j < kB; ++j) {
    v[b + j] = make_float4(0.f, 0.f, 0.f, 0.f);
    w[j][0] = w[j][1] = w[j][2] = w[j][3] = 0ull;
    const uint64_t* p = addr(b + j);
    if (p != nullptr) {
      ld_relaxed_v2(p, w[j][0], w[j][1], sys);
      ld_relaxed_v2(p + 2, w[j][2], w[j][3], sys);
      pending |= 1u << j;
    }
  }
  const bool ok = between();
  unsigned ns = 32;
  while (true) {
#pragma unroll
    for (int j = 0; j < kB; ++j)
      if (((pending >> j) & 1u) && all_tagged4(w[j][0], w[j][1], w[j][2], w[j][3], tag)) {
        v[b + j] = make_float4(word_value(w[j][0]), word_value(w[j][1]), word_value(w[j][2]), word_value(w[j][3]));
        pending &= ~(1u << j);
      }
    if (pending == 0) return ok;
    if (!ok || global_timer_ns() - t0 > kWaitLimitNs) return false;
    poll_backoff(ns);
#pragma unroll
    for (int j = 0; j < kB; ++j)
      if ((pending >> j) & 1u) {
        const uint64_t* p = addr(b + j);
        ld_relaxed_v2(p, w[j][0], w[j][1], sys);
        ld_relaxed_v2(p + 2, w[j][2], w[j][3], sys);
      }
  }
}

// Shared preparation: consumer thread t holds columns 4t + 4 kT j, j < J
// (the whole activation for n <= 4 kT kPre), read in batches of kBatch groups
// (load_tagged_batch); the wait prefix's polls run while the first batch is
// in flight.  False on a timeout or when `between` fails.
template <int kT, int J, int kMaxB, class Between>
__device__ __forceinline__ bool cta_x_load(const Op& op, const uint64_t* m, uint32_t tag, bool sys,
                                           float4 (&v)[J], const Between& between) {
  const int t = static_cast<int>(threadIdx.x);
  const int n = op.n;
  if (m == nullptr) {
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = 4 * kT * j + 4 * t;
      v[j] = c < n ? __ldcg(reinterpret_cast<const float4*>(op.x() + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    return between();
  }
  const uint64_t t0 = global_timer_ns();
  const auto addr = [&](int j) -> const uint64_t* {
    const int c = 4 * kT * j + 4 * t;
    return c < n ? m + c : nullptr;
  };
  constexpr int kB = J < kMaxB ? J : kMaxB;
  if (!load_tagged_batch<kB>(0, addr, tag, sys, t0, v, between)) return false;
#pragma unroll
  for (int b = kB; b < J; b += kB)
    if (4 * kT * b < n && !load_tagged_batch<kB>(b, addr, tag, sys, t0, v, NoPoll{})) return false;
  return true;
}

// RMSNorm of the held activation (the reference's rmsnorm_kernel,
// src/model_cuda_v2_shared.cu:74-89): ss = 1 / sqrt(sum(x^2) / n + 1e-5),
// x = weight * (ss * x).  The sum runs in one fixed order (per thread, the
// warp butterfly, warps in order), so every CTA normalises identically.
template <int kT, int J>
__device__ __forceinline__ void cta_rmsnorm(float4 (&v)[J], int n, const float* weight, float* red) {
  constexpr int kW = kT / 32;
  const int t = static_cast<int>(threadIdx.x);
  float ssq = 0.f;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    ssq = fmaf(v[j].x, v[j].x, ssq);
    ssq = fmaf(v[j].y, v[j].y, ssq);
    ssq = fmaf(v[j].z, v[j].z, ssq);
    ssq = fmaf(v[j].w, v[j].w, ssq);
  }
  ssq = warp_sum(ssq);
  if ((t & 31) == 0) red[t >> 5] = ssq;
  named_sync<kT>();
  float sum = red[0];
#pragma unroll
  for (int w = 1; w < kW; ++w) sum += red[w];
  const float ss = 1.0f / sqrtf(sum / static_cast<float>(n) + 1e-5f);
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = 4 * kT * j + 4 * t;
    if (c < n) {
      const float4 g = __ldg(reinterpret_cast<const float4*>(weight + c));
      v[j] = make_float4(g.x * (ss * v[j].x), g.y * (ss * v[j].y), g.z * (ss * v[j].z), g.w * (ss * v[j].w));
    }
  }
}

// W8A32 digit-pair planes and group factors (digit_quad) of the held activation
// into shared memory.
// kUnroll: the held values stay in registers; rolled (the kernels with the
// dependency code), they go through a per-thread local array instead, which
// keeps the prologue's registers below the row loop's.
template <int kT, bool kUnroll, int J>
__device__ __forceinline__ void cta_digits(const float4 (&v)[J], int n, int8_t* planes, float* fac) {
  const int lane = threadIdx.x & 31;
  if constexpr (kUnroll) {
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = 4 * kT * j + 4 * static_cast<int>(threadIdx.x);
      if (4 * kT * j < n) digit_quad(v[j], c < n, c, n, planes, fac, lane);  // CTA-uniform
    }
  } else {
#pragma unroll 1
    for (int j = 0; j < J; ++j) {
      const int c = 4 * kT * j + 4 * static_cast<int>(threadIdx.x);
      if (4 * kT * j < n) digit_quad(v[j], c < n, c, n, planes, fac, lane);  // CTA-uniform
    }
  }
}

// Fused W8A8: the quantised activation into shared memory, bit-identical to
// x_quant_prologue; from the held values when they cover n, else (an input
// ready at launch, n > 4 kT kPre) read a second time.
template <int kT, int J>
__device__ __forceinline__ float cta_quant(const float4 (&v)[J], const float* x, int n, int8_t* xq,
                                           float* red) {
  constexpr int kW = kT / 32;
  const int t = static_cast<int>(threadIdx.x);
  const bool hold = n <= 4 * kT * J;
  float m = 0.f;
  if (hold) {
#pragma unroll
    for (int j = 0; j < J; ++j)
      m = fmaxf(m, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
  } else {
    for (int c = 4 * t; c < n; c += 4 * kT) {
      const float4 u = __ldcg(reinterpret_cast<const float4*>(x + c));
      m = fmaxf(m, fmaxf(fmaxf(fabsf(u.x), fabsf(u.y)), fmaxf(fabsf(u.z), fabsf(u.w))));
    }
  }
  m = warp_max(m);
  if ((t & 31) == 0) red[t >> 5] = m;
  named_sync<kT>();
  float amax = red[0];
#pragma unroll
  for (int w = 1; w < kW; ++w) amax = fmaxf(amax, red[w]);
  const float scale = act_scale(amax);
  const float inv = 1.0f / scale;
  if (hold) {
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = 4 * kT * j + 4 * t;
      if (c < n) *reinterpret_cast<uint32_t*>(xq + c) = quant_quad(v[j], inv);
    }
  } else {
    for (int c = 4 * t; c < n; c += 4 * kT)
      *reinterpret_cast<uint32_t*>(xq + c) = quant_quad(__ldcg(reinterpret_cast<const float4*>(x + c)), inv);
  }
  return scale;
}

// Per-warp preparation (W8A32, when no two warps share a slice): the lane's
// chunks k = 0, 1 of its slice, 16 columns each at col0 + 512k, as
// v[4k + j] = columns col0 + 512k + 4j .. + 3, in batches of kB groups
// (load_tagged_batch); the wait prefix's polls run while the first is in
// flight.  False on a timeout or when `between` fails.
template <int kB, class Between>
__device__ __forceinline__ bool warp_x_load(const Op& op, const uint64_t* m, uint32_t tag, bool sys, int col0,
                                            unsigned vmask, float4 (&v)[kPre], const Between& between) {
  if (m == nullptr) {
#pragma unroll
    for (int k = 0; k < 2; ++k)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        v[4 * k + j] = ((vmask >> k) & 1u)
                           ? __ldcg(reinterpret_cast<const float4*>(op.x() + col0 + 512 * k + 4 * j))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
    return between();
  }
  const uint64_t t0 = global_timer_ns();
  const auto addr = [&](int q) -> const uint64_t* {
    return ((vmask >> (q >> 2)) & 1u) ? m + col0 + 512 * (q >> 2) + 4 * (q & 3) : nullptr;
  };
  static_assert(kPre % kB == 0, "whole batches");
  if (!load_tagged_batch<kB>(0, addr, tag, sys, t0, v, between)) return false;
#pragma unroll
  for (int b = kB; b < kPre; b += kB)
    if (!load_tagged_batch<kB>(b, addr, tag, sys, t0, v, NoPoll{})) return false;
  return true;
}

// The lane's digit pairs of chunks 0, 1 in registers (xd as load_digit_chunk
// lays them out).  The quad of lanes
// holding a group (group lane/4 + 8k of the slice) finds the group's max
// together, so digits and factors are exactly those of digit_quad.
__device__ __forceinline__ void warp_digits(const float4 (&v)[kPre], unsigned vmask, uint4 (&xd)[2][4],
                                            float (&fac)[2]) {
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 q = v[4 * k + j];
      m = fmaxf(m, fmaxf(fmaxf(fabsf(q.x), fabsf(q.y)), fmaxf(fabsf(q.z), fabsf(q.w))));
    }
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    const int e = static_cast<int>(__float_as_uint(m) >> 23);
    float scale_up, factor;
    if (e >= 13 && e <= 254) {
      scale_up = __uint_as_float(static_cast<uint32_t>(259 - e) << 23);
      factor = __uint_as_float(static_cast<uint32_t>(e - 12) << 23);
    } else if (e == 255) {
      scale_up = 0.f;
      factor = __uint_as_float(0x7fc00000u);
    } else {
      scale_up = 0.f;
      factor = 0.f;
    }
    // words[pair][w]: the pair plane's int16 values of columns 2w, 2w + 1
    uint32_t words[2][8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 q = v[4 * k + j];
      int a1, a2, b1, b2, c1, c2, d1, d2;
      digit_pairs(q.x * scale_up, a1, a2);
      digit_pairs(q.y * scale_up, b1, b2);
      digit_pairs(q.z * scale_up, c1, c2);
      digit_pairs(q.w * scale_up, d1, d2);
      words[0][2 * j] = pack16(a1, b1);
      words[0][2 * j + 1] = pack16(c1, d1);
      words[1][2 * j] = pack16(a2, b2);
      words[1][2 * j + 1] = pack16(c2, d2);
    }
    const bool valid = (vmask >> k) & 1u;
#pragma unroll
    for (int p = 0; p < 2; ++p)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t* w = words[p] + 4 * h;
        xd[k][2 * p + h] = valid ? make_uint4(w[0], w[1], w[2], w[3]) : make_uint4(0, 0, 0, 0);
      }
    fac[k] = valid ? factor : 0.f;
  }
}

// The activation prologue runs once per activation change.

// Shared preparation into shared memory: W8A32 digit-pair planes + group factors,
// or the fused W8A8 int8 copy (its scale into *xscale).  All consumer threads
// call it.  False (on every thread) when an input row did not arrive in time.
// J float4 of the activation per consumer thread (columns 4t + 4 kT j, j < J).
template <Form F, int kT, bool kUnroll, int J, class Between>
__device__ __forceinline__ bool prep_cta_j(const Op& op, const uint64_t* m, uint32_t tag, bool sys,
                                           unsigned char* xregion, float* red, float* red2, float* xscale,
                                           const Between& between) {
  float4 pre[J];
  bool fail = !cta_x_load<kT, J, F == Form::kW8A8Fused ? kPre : kBatch>(op, m, tag, sys, pre, between);
  fail = named_sync_or<kT>(fail);  // also: every consumer is done reading the shared region
  if (fail) return false;
  const int n = op.n;
  if (op.norm_w != nullptr) cta_rmsnorm<kT, J>(pre, n, op.norm_w, red2);
  if constexpr (F == Form::kW8A32) {
    int8_t* planes = reinterpret_cast<int8_t*>(xregion);
    cta_digits<kT, kUnroll || J <= 4, J>(pre, n, planes, reinterpret_cast<float*>(planes + 4 * n));
  } else {
    *xscale = cta_quant<kT, J>(pre, op.x(), n, reinterpret_cast<int8_t*>(xregion), red);
  }
  named_sync<kT>();
  return true;
}

// W8A32 activations of up to 4 kT * 4 columns hold only as many float4 per
// thread as they need, unrolled in registers; wider ones (and the kernels'
// rolled loops) take the full kPre.
template <Form F, int kT, bool kUnroll, class Between>
__device__ __forceinline__ bool prep_cta(const Op& op, const uint64_t* m, uint32_t tag, bool sys,
                                         unsigned char* xregion, float* red, float* red2, float* xscale,
                                         const Between& between) {
  if constexpr (F == Form::kW8A32) {
    if (op.n <= 4 * kT * 2)
      return prep_cta_j<F, kT, kUnroll, 2>(op, m, tag, sys, xregion, red, red2, xscale, between);
    if (op.n <= 4 * kT * 4)
      return prep_cta_j<F, kT, kUnroll, 4>(op, m, tag, sys, xregion, red, red2, xscale, between);
  }
  return prep_cta_j<F, kT, kUnroll, kPre>(op, m, tag, sys, xregion, red, red2, xscale, between);
}

// A consumer warp's role in an op: its slice, its rows of a stage, and the
// chunks of its lanes that fall inside the row.
template <Form F, int kW>
struct Role {
  int sl, wj, col0;
  bool on;
  unsigned vmask;
  __device__ Role(const Op& op, int warp, int lane) {
    constexpr int K = chunks_per_lane(F);
    const int S = op.S;
    sl = warp % S;
    wj = warp / S;
    on = wj < kW / S;
    const int g_slice = min(8 * K, op.G() - sl * 8 * K);
    vmask = 0;
#pragma unroll
    for (int k = 0; k < K; ++k)
      if (on && (lane >> 2) + 8 * k < g_slice) vmask |= 1u << k;
    col0 = sl * slice_cols(F) + 16 * lane;
  }
};

// Warps 0 .. kW-1 consume (kRB rows per warp per stage), warp kW is the
// producer (bulk copies).
// kTags: some op reads another op's rows (mirrors, tags, polls, peers); a
// chain without dependencies runs a kernel compiled without any of it.
template <Form F, int kW, int kRB, bool kEpi, bool kTags>
__global__ void __launch_bounds__((kW + 1) * 32, 1) gemv_chain_kernel(const Args a) {
  constexpr int kT = kW * 32;  // consumer threads
  extern __shared__ __align__(1024) unsigned char smem[];
  Smem sm(smem);
  unsigned char* ring = smem + a.ring_off;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grid = static_cast<int>(gridDim.x);
  const int cta = static_cast<int>(blockIdx.x);

  if (threadIdx.x == 0) {
    for (int i = 0; i < a.ring; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.free[i], 1);
      sm.counters[i] = 0;
    }
    *sm.broken = 0;
    *sm.last_cta = 0;
    *sm.issued = 0;
    *sm.seq = __ldcg(a.seq);
    fence_barrier_init();
  }
  if (a.table_off != 0) {
    const uint4* src = reinterpret_cast<const uint4*>(a.ops);
    uint4* dst = reinterpret_cast<uint4*>(smem + a.table_off);
    constexpr int kOpVecs = static_cast<int>(sizeof(Op) / sizeof(uint4));
    for (int i = threadIdx.x; i < a.count * kOpVecs; i += blockDim.x) dst[i] = __ldg(src + i);
    int* pdst = reinterpret_cast<int*>(smem + a.table_off + sizeof(Op) * a.count);
    for (int i = threadIdx.x; i <= a.n_phases; i += blockDim.x) pdst[i] = __ldg(a.phases + i);
    for (int i = threadIdx.x; i < a.n_polls; i += blockDim.x) pdst[a.n_phases + 1 + i] = __ldg(a.polls + i);
  }
  __syncthreads();
  const Op* ops = a.table_off != 0 ? reinterpret_cast<const Op*>(smem + a.table_off) : a.ops;
  const int* phases =
      a.table_off != 0 ? reinterpret_cast<const int*>(smem + a.table_off + sizeof(Op) * a.count) : a.phases;
  const int* polls = a.table_off != 0 ? phases + a.n_phases + 1 : a.polls;
  const int cnt = cta_units(phases, a.n_phases, cta, grid);
  const unsigned seq = *sm.seq;

  if (warp == kW) {
    // ---- producer: unit i into slot i % ring once the consumers freed it
    if (lane == 0) {
      int o = 0;
      Cursor cur(phases, a.n_phases, cta, grid);
      for (int i = 0; i < cnt; ++i, cur.next()) {
        const int slot = i % a.ring;
        if (i >= a.ring && !mbar_wait_bounded(&sm.free[slot], ((i / a.ring) - 1) & 1, kWaitLimitNs)) {
          record_error(a, kDevStageTimeout);
          *sm.broken = 1;
        }
        if (*sm.broken) break;
        o = find_op(ops, a.count, cur.u, o);
        fence_proxy_async_smem();  // consumers' reads of the slot precede the copy's writes
        issue_unit<kEpi>(a, ops, ring, sm.full, o, cur.u, slot);
        *sm.issued = i + 1;
      }
    }
  } else {
    constexpr int K = chunks_per_lane(F);
    constexpr int kSlice = slice_cols(F);
    constexpr int kLanesPerRow = 32 / kRB;
    int o = 0, cur = -1, known = 0, epoch = -1;
    int n = 0, d = 0, Gr = 0, S = 1, R = 0, Ru = 0, epi = kEpiStore, base = 0;
    float* y = nullptr;
    int sl = 0, wj = 0;
    bool warp_on = false;
    unsigned vmask = 0;
    float xscale = 0.f;
    uint4 xd[2][4];  // W8A32 digit pairs of chunks 0, 1 (load_digit_chunk)
    float fac[2];
    uint4 xv[4];     // W8A8 int8 chunks 0..3

    Cursor it(phases, a.n_phases, cta, grid);
    for (int i = 0; i < cnt; ++i, it.next()) {
      const int u = it.u;
      o = find_op(ops, a.count, u, o);
      if (o != cur) {
        const Op& op = ops[o];
        const int wait = op.wait, ep = op.epoch;
        bool fail = false;
        // once a wait has expired in this CTA, later ops wait for nothing
        // (their rows are not produced): the launch ends in bounded time
        const bool broken = *sm.broken != 0;
        // ops of the wait prefix that the activation's producer does not imply;
        // polled while the activation's own loads are in flight when it changes
        const bool need_poll = kTags && wait > known && op.poll_count > 0;  // CTA-uniform
        const bool do_poll = need_poll && !broken;
        const PrefixPoll<kT> prefix{a, ops, polls, op.poll_first, op.poll_count, seq, do_poll};
        bool polled = false;
        n = op.n; d = op.d; Gr = op.G(); R = op.R; base = op.unit_base; y = op.y;
        if constexpr (kEpi) {
          Ru = op.Ru();
          epi = op.epi;
        } else {
          Ru = R;
        }
        if (ep != epoch) {
          epoch = ep;
          const Role<F, kW> role(op, warp, lane);
          S = op.S; sl = role.sl; wj = role.wj; warp_on = role.on; vmask = role.vmask;
          const int col0 = role.col0;
          // (a broken CTA reads the activation as it stands, without waiting)
          const uint64_t* src_m =
              kTags && op.src >= 0 && !broken ? a.mirror + mirror_half(a, seq) + ops[op.src].mirror : nullptr;
          const uint32_t src_tag = row_tag(seq, op.src);
          // No warp polls while another still computes on this SM: the
          // consumers first finish their units of the previous phase (the
          // activation needs their rows anyway), and they start the new op
          // together once it has arrived.
          const bool gate = kTags && (op.src >= 0 || need_poll);  // CTA-uniform
          if (gate) named_sync<kT>();
          if constexpr (F == Form::kW8A8) {
            xscale = __ldcg(op.xs);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              xv[k] = ((vmask >> k) & 1u)
                          ? __ldcg(reinterpret_cast<const uint4*>(op.xq() + col0 + 512 * k))
                          : make_uint4(0, 0, 0, 0);
          } else if (F == Form::kW8A32 && op.S == kW && op.norm_w == nullptr) {
            // every warp owns its slice: prepare it in registers, no barrier
            float4 pre[kPre];
            // (one batch of loads, except in the narrow-row kernels, whose
            // registers leave room for half of it)
            if (!warp_x_load<kRB == 8 ? kPre : kBatch>(op, src_m, src_tag, a.world > 1, col0, vmask, pre, prefix))
              fail = true;
            if (gate) fail = named_sync_or<kT>(fail);
            polled = true;
            if constexpr (F == Form::kW8A32) warp_digits(pre, vmask, xd, fac);
          } else {
            float t_scale = 0.f;
            if (!prep_cta<F, kT, !kTags>(op, src_m, src_tag, a.world > 1, smem + a.x_off, sm.red, sm.red2, &t_scale,
                                         prefix))
              fail = true;
            polled = true;
            xscale = t_scale;
            if constexpr (F == Form::kW8A32) {
              const int8_t* planes = reinterpret_cast<const int8_t*>(smem + a.x_off);
              const float* facs = reinterpret_cast<const float*>(planes + 4 * n);
#pragma unroll
              for (int k = 0; k < 2; ++k) {
                const bool v = (vmask >> k) & 1u;
                if (v) {
                  load_digit_chunk(planes, n, col0 + 512 * k, xd[k]);
                } else {
#pragma unroll
                  for (int p = 0; p < 4; ++p) xd[k][p] = make_uint4(0, 0, 0, 0);
                }
                fac[k] = v ? facs[(col0 + 512 * k) >> 6] : 0.f;
              }
            } else {
              const int8_t* q8 = reinterpret_cast<const int8_t*>(smem + a.x_off);
#pragma unroll
              for (int k = 0; k < 4; ++k)
                xv[k] = ((vmask >> k) & 1u) ? *reinterpret_cast<const uint4*>(q8 + col0 + 512 * k)
                                            : make_uint4(0, 0, 0, 0);
            }
          }
        }
        if (need_poll && !polled) {
          if (do_poll) fail = !poll_ops<kT>(a, ops, polls, op.poll_first, op.poll_count, seq) || fail;
          fail = named_sync_or<kT>(fail);
        }
        if (fail) {
          record_error(a, kDevChainTimeout);
          *sm.broken = 1;
        }
        if (wait > known) known = wait;
        cur = o;
      }
      const int slot = i % a.ring;
      const int row0 = (u - base) * Ru;
      const int rows = min(Ru, d - row0);
      bool ok = !*sm.broken;
      if (ok && !mbar_wait_bounded(&sm.full[slot], (i / a.ring) & 1, kWaitLimitNs)) {
        record_error(a, kDevStageTimeout);
        *sm.broken = 1;
        ok = false;
      }
      ok = __all_sync(0xffffffffu, ok);
      const int8_t* wst = reinterpret_cast<const int8_t*>(ring + static_cast<size_t>(slot) * a.slot_bytes);
      const float* sst = reinterpret_cast<const float*>(wst + static_cast<size_t>(R) * n);
      float* part = reinterpret_cast<float*>(smem + a.part_off) + slot * a.part_stride;
      if (ok && warp_on) {
        const int j0 = wj * kRB;
        // a SwiGLU stage holds the gate's rows [0, Ru) and the up's [Ru, R)
        const int nvalid = (kEpi && epi == kEpiSwiglu && j0 >= Ru ? Ru + rows : rows) - j0;
        if (nvalid > 0) {
          const int8_t* wr = wst + static_cast<size_t>(j0) * n + sl * kSlice;
          const float* sr = sst + j0 * Gr + sl * 8 * K;
          float v[kRB];
          if constexpr (F == Form::kW8A32)
            rows_w8a32<kRB>(wr, sr, n, Gr, nvalid, xd, fac, vmask, lane, v);
          else
            rows_w8a8<kRB>(wr, sr, n, Gr, nvalid, xv, vmask, lane, xscale, v);
          const float total = warp_sum_rows<kRB>(v, lane);
          const int r = lane / kLanesPerRow;
          if ((lane & (kLanesPerRow - 1)) == 0 && r < nvalid) part[(j0 + r) * S + sl] = total;
        }
      }
      // The last warp to finish with this slot sums the slices of its rows in
      // slice order, stores them (into y and, tagged, into the op's mirror)
      // and frees the slot.
      __syncwarp();
      int last = 0;
      if (lane == 0) {
        __threadfence_block();
        last = atomicAdd(&sm.counters[slot], 1) == kW - 1;
        if (last) sm.counters[slot] = 0;
        __threadfence_block();
      }
      if (__shfl_sync(0xffffffffu, last, 0)) {
        if (!*sm.broken) {
          // the op's mirror and the ADD base, from the table (kept out of the
          // registers of the row loop)
          const Op& op = ops[o];
          // rows r of the op are words row_off + r of its mirror (the whole GEMV's rows)
          const uint32_t half = mirror_half(a, seq);
          const size_t my_off = kTags && op.mirror >= 0 ? half + op.mirror + op.row_off : 0;
          const bool share = kTags && a.world > 1;
          uint64_t* my_mirror = kTags && op.mirror >= 0 ? a.mirror + my_off : nullptr;
          const uint32_t my_tag = row_tag(seq, o);
          const uint64_t* base_mirror =
              kTags && op.base >= 0 ? a.mirror + half + ops[op.base].mirror + op.row_off : nullptr;
          const uint32_t base_tag = row_tag(seq, op.base);
          bool late = false;
          const uint64_t t0 = global_timer_ns();
          for (int rr = lane; rr < rows; rr += 32) {
            float v = part[rr * S];
            for (int s2 = 1; s2 < S; ++s2) v += part[rr * S + s2];
            if (kEpi && epi == kEpiSwiglu) {
              const int ru = Ru + rr;
              float up = part[ru * S];
              for (int s2 = 1; s2 < S; ++s2) up += part[ru * S + s2];
              v *= (1.0f / (1.0f + expf(-v)));
              v *= up;
            } else if (kEpi && epi == kEpiAdd) {
              float b;
              if (base_mirror != nullptr && !*sm.broken) {
                uint64_t w = ld_relaxed_b64(base_mirror + row0 + rr, share);
                unsigned ns = 32;
                while (!has_tag(w, base_tag) && !late) {
                  late = global_timer_ns() - t0 > kWaitLimitNs;
                  poll_backoff(ns);
                  w = ld_relaxed_b64(base_mirror + row0 + rr, share);
                }
                b = word_value(w);
              } else {
                b = __ldcg(y + row0 + rr);
              }
              v = b + v;
            }
            y[row0 + rr] = v;
            if (my_mirror != nullptr) {
              const uint64_t w = tagged(v, my_tag);
              if (share) {
                // every rank's mirror, over NVLink (plain peer stores)
                for (int pr = 0; pr < a.world; ++pr)
                  st_relaxed_sys_b64(reinterpret_cast<unsigned long long*>(a.peers[pr] + my_off + row0 + rr), w);
              } else {
                st_relaxed_b64(my_mirror + row0 + rr, w);
              }
            }
          }
          if (late) {
            record_error(a, kDevChainTimeout);
            *sm.broken = 1;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.free[slot]);
      }
    }
  }

  __syncthreads();
  if (threadIdx.x == kW * 32) {
    // After an error, copies still in flight land before the CTA exits.
    const int iss = *sm.issued;
    for (int s = 0; s < a.ring && s < iss; ++s) {
      const int last_i = s + ((iss - 1 - s) / a.ring) * a.ring;
      mbar_wait_bounded(&sm.full[s], (last_i / a.ring) & 1, kWaitLimitNs);
    }
    __threadfence();
    *sm.last_cta = atomicAdd(a.finished, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  // The last CTA advances the launch sequence for the next launch: every
  // other CTA has read this launch's value and left its loops.
  if (*sm.last_cta && threadIdx.x == 0) {
    *a.finished = 0;
    *a.seq = seq % kSeqPeriod + 1;
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Kernel shape: consumer warps per CTA, rows per warp per stage, CTAs per SM.
struct Variant {
  int warps, rb, per_sm;
  bool epi;   // some op has a non-store epilogue: the kernel with epilogue code
  bool tags;  // some op reads another op's rows: the kernel with mirror code
};

struct Plan {
  std::vector<Op> ops;
  std::vector<int> phases;  // first unit of every phase, then the unit count
  std::vector<int> polls;   // ops checked by tag, per op a run (Op::poll_first)
  size_t mirror_words = 0;
  Args args = {};
  Variant v = {};
  size_t smem = 0;
  int grid = 0;
  int epochs = 0;
};

bool overlaps(const void* a, size_t an, const void* b, size_t bn) {
  const uintptr_t pa = reinterpret_cast<uintptr_t>(a), pb = reinterpret_cast<uintptr_t>(b);
  return pa < pb + bn && pb < pa + an;
}

// The kernel shape for a chain of `form`: 8 consumer warps of 8 (W8A32) or
// 4 (W8A8) rows each -- 64 row slices of 1024 columns (W8A32) or 32 of 2048
// (W8A8) in flight per SM.  Launch flags bit 8 halves the rows per warp (for
// comparisons).
Variant pick_variant(int form, unsigned flags) {
  const bool a32 = form == 0;
  if (flags & (1u << 8)) return {8, a32 ? 4 : 2, 1, false, false};
  return {8, a32 ? 8 : 4, 1, false, false};
}

// The activation held by the consumers (4 kT kPre columns) bounds ops that
// prepare the whole vector in shared memory.
constexpr int kMaxHeldCols = 4 * 8 * 32 * kPre;

// Validates the op list and lays out the chain.  Returns MLI_OK,
// MLI_ERR_INVALID_ARG or MLI_ERR_UNSUPPORTED (without touching the device).
// row_offset / d_total (NULL: 0 / d): op i computes rows [row_offset[i],
// row_offset[i] + d) of a GEMV of d_total[i] rows, its y pointing at the first
// of them; an op reading the whole vector takes the full buffer
// (y - row_offset) as its x, and its rows arrive through the producer's
// mirror from every rank.
int plan_chain(const mli_gemv_op* in, int count, int sm_count, int smem_per_sm, int smem_optin,
               unsigned flags, const int* row_offset, const int* d_total, Plan* p) {
  if (!in || count <= 0 || sm_count <= 0 || smem_optin <= 0 || smem_per_sm <= 0)
    return MLI_ERR_INVALID_ARG;
  if (count > kMaxOps) return MLI_ERR_UNSUPPORTED;
  const int form = in[0].form;
  if (form < 0 || form > 2) return MLI_ERR_INVALID_ARG;
  const Form f = static_cast<Form>(form);
  Variant var = pick_variant(form, flags);
  for (int i = 0; i < count; ++i) var.epi |= in[i].epilogue != kEpiStore;
  p->v = var;
  p->ops.assign(count, Op{});
  p->phases.clear();
  p->polls.clear();
  std::vector<char> is_comp(count, 0);  // op i is the up projection of the SwiGLU pair at i - 1
  int max_wait = -1;
  long long units = 0;
  size_t slot = 0, xbytes = 0, mirror = 0;
  int part_stride = 0, epoch = -1;
  auto roff = [&](int i) { return row_offset ? row_offset[i] : 0; };
  auto dtot = [&](int i) { return d_total ? d_total[i] : in[i].d; };
  for (int i = 0; i < count; ++i) {
    const mli_gemv_op& s = in[i];
    const bool companion = i > 0 && in[i - 1].epilogue == kEpiSwiglu && !is_comp[i - 1];
    if (roff(i) < 0 || static_cast<long long>(roff(i)) + s.d > dtot(i)) return MLI_ERR_INVALID_ARG;
    if (companion && (roff(i) != roff(i - 1) || dtot(i) != dtot(i - 1))) return MLI_ERR_INVALID_ARG;
    is_comp[i] = companion;
    if (s.form != form) return MLI_ERR_INVALID_ARG;
    if (s.epilogue < kEpiStore || s.epilogue > kEpiSwiglu) return MLI_ERR_INVALID_ARG;
    if (companion) {
      // same activation, norm, shape and dependencies as its gate; no output of its own
      const mli_gemv_op& g = in[i - 1];
      if (s.epilogue != kEpiStore || s.n != g.n || s.d != g.d || s.wait != g.wait || s.x != g.x ||
          s.xq != g.xq || s.xs != g.xs || s.norm_w != g.norm_w)
        return MLI_ERR_INVALID_ARG;
    } else if (!s.y) {
      return MLI_ERR_INVALID_ARG;
    }
    if (s.epilogue == kEpiSwiglu && i + 1 >= count) return MLI_ERR_INVALID_ARG;
    if (!s.w_q || !s.w_s || s.n <= 0 || s.d <= 0 || s.group_size <= 0) return MLI_ERR_INVALID_ARG;
    if (f == Form::kW8A8 ? (!s.xq || !s.xs) : !s.x) return MLI_ERR_INVALID_ARG;
    if (s.wait < 0 || s.wait > i) return MLI_ERR_INVALID_ARG;
    if (!companion && f != Form::kW8A8 && overlaps(s.y, 4u * s.d, s.x, 4u * s.n)) return MLI_ERR_INVALID_ARG;
    if (s.norm_w != nullptr && f == Form::kW8A8) return MLI_ERR_INVALID_ARG;  // int8 input: nothing to norm
    if (s.group_size != kGroup || s.n % 256 != 0) return MLI_ERR_UNSUPPORTED;
    if (!aligned(s.w_q, 16) || !aligned(s.w_s, 16) ||
        !aligned(f == Form::kW8A8 ? static_cast<const void*>(s.xq) : s.x, 16) ||
        (s.norm_w != nullptr && !aligned(s.norm_w, 16)))
      return MLI_ERR_UNSUPPORTED;
    Op& op = p->ops[i];
    op.y = s.y;
    op.act = f == Form::kW8A8 ? static_cast<const void*>(s.xq) : static_cast<const void*>(s.x);
    op.xs = s.xs;
    op.w = s.w_q;
    op.s = s.w_s;
    op.norm_w = s.norm_w;
    op.n = s.n;
    op.d = s.d;
    op.row_off = roff(i);
    op.d_total = dtot(i);
    const int S = (s.n + slice_cols(f) - 1) / slice_cols(f);
    if (S > kMaxSlices) return MLI_ERR_UNSUPPORTED;
    // the whole vector is prepared in shared memory when some warps share a
    // slice or a norm needs the whole row
    const bool shared_prep = f == Form::kW8A8Fused || (f == Form::kW8A32 && (S < var.warps || s.norm_w));
    const int R = var.rb * (var.warps / S);
    op.S = static_cast<uint8_t>(S);
    op.R = static_cast<uint16_t>(R);
    op.epi = static_cast<uint8_t>(companion ? kEpiCompanion : s.epilogue);
    // a SwiGLU stage holds R/2 gate rows and their R/2 up rows: a warp's rows
    // must fall in one half
    if (op.epi == kEpiSwiglu && (R / 2) % var.rb != 0) return MLI_ERR_UNSUPPORTED;
    const int n_stages = companion ? 0 : (s.d + op.Ru() - 1) / op.Ru();
    op.unit_base = static_cast<int>(units);
    if (s.wait > max_wait) {  // a new dependency: a new phase
      p->phases.push_back(op.unit_base);
      max_wait = s.wait;
    }
    units += n_stages;
    if (units > (1ll << 30)) return MLI_ERR_UNSUPPORTED;
    op.wait = s.wait;
    // The activation's producer: the latest earlier op writing the buffer this
    // op reads (fp32 activations only; nothing in a chain writes int8).  It
    // must lie in the wait prefix, and the reader takes its rows from the
    // producer's mirror.
    op.src = -1;
    if (f != Form::kW8A8) {
      for (int j = i - 1; j >= 0; --j)
        if (!is_comp[j] && in[j].y - roff(j) == s.x) {
          op.src = j;
          break;
        }
      if (op.src >= 0 && (op.src >= s.wait || dtot(op.src) != s.n)) return MLI_ERR_INVALID_ARG;
      if (companion) op.src = p->ops[i - 1].src;
    }
    // More columns than the consumers hold: only an input ready at launch,
    // without a norm, can be read a second time (fused W8A8 quantisation).
    if (shared_prep && s.n > kMaxHeldCols && !(f == Form::kW8A8Fused && op.src < 0 && s.norm_w == nullptr))
      return MLI_ERR_UNSUPPORTED;
    // The ADD epilogue's base: the latest earlier op writing the same y.
    op.base = -1;
    if (s.epilogue == kEpiAdd) {
      for (int j = i - 1; j >= 0; --j)
        if (!is_comp[j] && in[j].y == s.y) {
          op.base = j;
          break;
        }
      if (op.base >= 0 && (op.base >= s.wait || in[op.base].d != s.d || roff(op.base) != roff(i) ||
                           dtot(op.base) != dtot(i)))
        return MLI_ERR_INVALID_ARG;
    }
    op.mirror = -1;  // assigned below to the ops some later op reads
    // Ops of the wait prefix [0, wait) that must be checked by tag: all but
    // those implied by an op whose rows this op reads anyway (that op was
    // written only after its own prefix [0, wait_j) had completed).  A
    // SwiGLU pair completes together.
    op.poll_first = static_cast<int>(p->polls.size());
    {
      int prefix = 0;  // ops [0, prefix) implied
      std::vector<int> implied;
      auto imply = [&](int j) {
        const int g = is_comp[j] ? j - 1 : j;
        implied.push_back(g);
        if (!is_comp[g] && in[g].epilogue == kEpiSwiglu) implied.push_back(g + 1);
        if (in[g].wait > prefix) prefix = in[g].wait;
      };
      if (op.src >= 0) imply(op.src);
      if (op.base >= 0) imply(op.base);
      for (int j = s.wait - 1; j >= prefix; --j) {
        bool done = false;
        for (int k : implied) done |= k == j;
        if (done) continue;
        const int g = is_comp[j] ? j - 1 : j;
        p->polls.push_back(g);
        imply(g);
      }
    }
    op.poll_count = static_cast<int>(p->polls.size()) - op.poll_first;
    // Same activation as the previous op, with the same prefix to wait for:
    // the CTA keeps its prepared copy.
    const bool same = i > 0 && s.n == in[i - 1].n && s.wait == in[i - 1].wait && s.norm_w == in[i - 1].norm_w &&
                      op.src == p->ops[i - 1].src &&
                      (f == Form::kW8A8 ? (s.xq == in[i - 1].xq && s.xs == in[i - 1].xs)
                                        : s.x == in[i - 1].x);
    if (!same) ++epoch;
    op.epoch = epoch;
    const size_t stage = static_cast<size_t>(R) * s.n + static_cast<size_t>(R) * op.G() * 4u;
    if (stage > slot) slot = stage;
    // shared activation region: fused W8A8 its int8 copy; W8A32 its digit
    // planes and group factors when prepared per CTA
    const size_t xb = f == Form::kW8A8Fused ? static_cast<size_t>(s.n)
                      : (f == Form::kW8A32 && shared_prep) ? 4u * s.n + op.G() * 4u : 0u;
    if (xb > xbytes) xbytes = xb;
    if (R * S > part_stride) part_stride = R * S;
  }
  p->phases.push_back(static_cast<int>(units));
  // Mirrors only for ops whose rows another op reads (as its activation, as
  // its ADD base, or to check completion): a chain without dependencies
  // writes none.
  std::vector<char> read(count, 0);
  for (int i = 0; i < count; ++i) {
    if (p->ops[i].src >= 0) read[p->ops[i].src] = 1;
    if (p->ops[i].base >= 0) read[p->ops[i].base] = 1;
  }
  for (int j : p->polls) read[j] = 1;
  // a row-sharded chain keeps every op's whole rows (its outputs are read back
  // from the mirrors)
  if (row_offset) std::fill(read.begin(), read.end(), 1);
  for (int i = 0; i < count; ++i)
    if (read[i] && p->ops[i].epi != kEpiCompanion) {
      p->ops[i].mirror = static_cast<int>(mirror);
      mirror += align_up(static_cast<size_t>(p->ops[i].d_total), 2);  // 16-byte aligned runs
      if (mirror > (1u << 30)) return MLI_ERR_UNSUPPORTED;
    }
  p->mirror_words = mirror;
  p->v.tags = mirror > 0 || !p->polls.empty() || row_offset != nullptr;
  Args& a = p->args;
  a.count = count;
  a.n_phases = static_cast<int>(p->phases.size()) - 1;
  a.n_polls = static_cast<int>(p->polls.size());
  a.units = static_cast<int>(units);
  a.slot_bytes = static_cast<uint32_t>(align_up(slot, 128));
  a.part_stride = part_stride;
  const size_t budget = var.per_sm == 1 ? static_cast<size_t>(smem_optin)
                                        : static_cast<size_t>(smem_per_sm) / var.per_sm - 1024;
  const size_t per_slot = a.slot_bytes + static_cast<size_t>(part_stride) * 4u;
  // Layout: header | tables (when they fit) | activation region | ring | partials.
  auto ring_for = [&](size_t table) -> int {
    const size_t ring_off = align_up(kHeader + table + xbytes, 128);
    if (budget <= ring_off) return 0;
    const size_t r = (budget - ring_off) / per_slot;
    return static_cast<int>(r < kMaxRing ? r : kMaxRing);
  };
  const size_t table =
      align_up(sizeof(Op) * count + sizeof(int) * (p->phases.size() + p->polls.size()), 128);
  const int ring_global = ring_for(0), ring_shared = ring_for(table);
  // Keep the tables in shared memory unless that costs a ring slot the chain
  // needs (three slots keep the stream going across an op switch).
  const bool shared_table = table <= 16384 && ring_shared >= (ring_global < 3 ? ring_global : 3);
  a.table_off = shared_table ? kHeader : 0u;
  a.x_off = static_cast<uint32_t>(kHeader + (shared_table ? table : 0));
  a.ring_off = static_cast<uint32_t>(align_up(a.x_off + xbytes, 128));
  const int ring = shared_table ? ring_shared : ring_global;
  if (ring < 2) return MLI_ERR_UNSUPPORTED;
  a.ring = ring;
  a.part_off = static_cast<uint32_t>(a.ring_off + static_cast<size_t>(ring) * a.slot_bytes);
  p->smem = a.part_off + static_cast<size_t>(ring) * part_stride * 4u;
  p->grid = var.per_sm * sm_count;  // every CTA resident (cooperative launch)
  p->epochs = epoch + 1;
  return MLI_OK;
}

using KernelFn = void (*)(const Args);

template <Form F, bool kEpi, bool kTags>
KernelFn kernel_shape(const Variant& v) {
  if constexpr (F == Form::kW8A32)
    return v.rb == 8 ? gemv_chain_kernel<F, 8, 8, kEpi, kTags> : gemv_chain_kernel<F, 8, 4, kEpi, kTags>;
  else
    return v.rb == 4 ? gemv_chain_kernel<F, 8, 4, kEpi, kTags> : gemv_chain_kernel<F, 8, 2, kEpi, kTags>;
}

// Three kernels per shape: no epilogue and no dependencies, dependencies
// without epilogues, epilogues (with or without dependencies).
template <Form F>
KernelFn kernel_epi(const Variant& v) {
  if (v.epi) return kernel_shape<F, true, true>(v);
  return v.tags ? kernel_shape<F, false, true>(v) : kernel_shape<F, false, false>(v);
}

KernelFn kernel_for(int form, const Variant& v) {
  switch (form) {
    case 0: return kernel_epi<Form::kW8A32>(v);
    case 1: return kernel_epi<Form::kW8A8>(v);
    default: return kernel_epi<Form::kW8A8Fused>(v);
  }
}

}  // namespace chain
}  // namespace mli

struct mli_chain {
  int device;
  int form;
  size_t smem;
  int grid;
  int threads;
  int world;         // ranks the chain's rows are shared with (1: none)
  bool peers_ready;  // sharded chains: mli_chain_set_peers has run
  mli::chain::KernelFn kernel;
  mli::chain::Args args;
  std::vector<mli::chain::Op> ops;  // host copy of the op table (mirror offsets, row ranges)
  void* dev_mem;     // op table, phases, polls, peer pointers, then the launch words
  void* mirror_mem;  // the mirrors (their own allocation, so that other ranks can map them)
  size_t mirror_bytes;
};

using namespace mli;

namespace {

int chain_create(const mli_gemv_op* ops, const int* row_offset, const int* d_total, int count, int world,
                 mli_chain** chain_out) {
  if (!chain_out) return set_status(MLI_ERR_INVALID_ARG);
  *chain_out = nullptr;
  if (!ops || count <= 0 || world < 1 || world > chain::kMaxPeers) return set_status(MLI_ERR_INVALID_ARG);
  cudaError_t err = cudaSuccess;
  const DeviceInfo& dev = current_device(&err);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  chain::Plan p;
  const int rc = chain::plan_chain(ops, count, dev.sm_count, dev.smem_per_sm, dev.smem_optin_per_cta,
                                   launch_flags(), row_offset, d_total, &p);
  if (rc != MLI_OK) return set_status(rc);
  const chain::KernelFn kfn = chain::kernel_for(ops[0].form, p.v);
  const int threads = (p.v.warps + 1) * 32;
  err = ensure_dynamic_smem(reinterpret_cast<const void*>(kfn), p.smem);
  if (err != cudaSuccess) return check_cuda(err);
  int per_sm = 0;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, threads, p.smem);
  if (err != cudaSuccess) return check_cuda(err);
  if (per_sm < p.v.per_sm) return set_status(MLI_ERR_UNSUPPORTED);
  // device block: op table | phases | polls | peer pointers | launch sequence, finished count
  const size_t table = chain::align_up(sizeof(chain::Op) * count, 256);
  const size_t phases = chain::align_up(sizeof(int) * p.phases.size(), 256);
  const size_t polls = chain::align_up(sizeof(int) * (p.polls.size() + 1), 256);
  const size_t peers = chain::align_up(sizeof(uint64_t*) * chain::kMaxPeers, 256);
  const size_t words = 256;
  // mirrors: one copy, or two (alternating by launch) when rows are shared
  const size_t half_words = chain::align_up(p.mirror_words, 32);
  const size_t mirror_bytes = chain::align_up(sizeof(uint64_t) * half_words * (world > 1 ? 2 : 1), 256) + 256;
  void* mem = nullptr;
  void* mir = nullptr;
  err = cudaMalloc(&mem, table + phases + polls + peers + words);
  if (err == cudaSuccess) err = cudaMalloc(&mir, mirror_bytes);
  if (err != cudaSuccess) {
    if (mem) cudaFree(mem);
    return set_status(MLI_ERR_CUDA, err);
  }
  char* base = static_cast<char*>(mem);
  err = cudaMemcpy(base, p.ops.data(), sizeof(chain::Op) * count, cudaMemcpyHostToDevice);
  if (err == cudaSuccess)
    err = cudaMemcpy(base + table, p.phases.data(), sizeof(int) * p.phases.size(), cudaMemcpyHostToDevice);
  if (err == cudaSuccess && !p.polls.empty())
    err = cudaMemcpy(base + table + phases, p.polls.data(), sizeof(int) * p.polls.size(),
                     cudaMemcpyHostToDevice);
  // zeroed mirrors carry tag 0, which no launch uses; the sequence starts at 1
  if (err == cudaSuccess) err = cudaMemset(mir, 0, mirror_bytes);
  if (err == cudaSuccess) err = cudaMemset(base + table + phases + polls, 0, peers + words);
  const unsigned first_seq = 1;
  if (err == cudaSuccess)
    err = cudaMemcpy(base + table + phases + polls + peers, &first_seq, sizeof(first_seq), cudaMemcpyHostToDevice);
  if (err != cudaSuccess) {
    cudaFree(mem);
    cudaFree(mir);
    return set_status(MLI_ERR_CUDA, err);
  }
  mli_chain* c = new mli_chain;
  c->device = dev.device;
  c->form = ops[0].form;
  c->smem = p.smem;
  c->grid = p.grid;
  c->threads = threads;
  c->world = world;
  c->peers_ready = world == 1;
  c->kernel = kfn;
  c->args = p.args;
  c->ops = p.ops;
  c->args.ops = reinterpret_cast<const chain::Op*>(base);
  c->args.phases = reinterpret_cast<const int*>(base + table);
  c->args.polls = reinterpret_cast<const int*>(base + table + phases);
  c->args.peers = reinterpret_cast<uint64_t* const*>(base + table + phases + polls);
  c->args.world = 1;  // rows are shared once every rank's mirror is known
  c->args.mirror = static_cast<uint64_t*>(mir);
  c->args.mirror_half = world > 1 ? static_cast<uint32_t>(half_words) : 0u;
  c->args.seq = reinterpret_cast<unsigned*>(base + table + phases + polls + peers);
  c->args.finished = c->args.seq + 1;
  c->args.err = device_error_word();
  c->dev_mem = mem;
  c->mirror_mem = mir;
  c->mirror_bytes = mirror_bytes;
  *chain_out = c;
  return set_status(MLI_OK);
}

}  // namespace

extern "C" {

int mli_chain_create(const mli_gemv_op* ops, int count, mli_chain** chain_out) {
  return chain_create(ops, nullptr, nullptr, count, 1, chain_out);
}

int mli_chain_create_sharded(const mli_gemv_op* ops, const int* row_offset, const int* d_total, int count,
                             int world, mli_chain** chain_out) {
  if (!row_offset || !d_total) {
    if (chain_out) *chain_out = nullptr;
    return set_status(MLI_ERR_INVALID_ARG);
  }
  return chain_create(ops, row_offset, d_total, count, world, chain_out);
}

int mli_chain_export(mli_chain* chain, unsigned char* ipc_handle) {
  if (!chain || !ipc_handle) return set_status(MLI_ERR_INVALID_ARG);
  cudaIpcMemHandle_t h;
  const cudaError_t err = cudaIpcGetMemHandle(&h, chain->mirror_mem);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(ipc_handle, &h, sizeof(h));
  return set_status(MLI_OK);
}

int mli_chain_set_peers(mli_chain* chain, void* const* peer_mirrors, int rank) {
  if (!chain || !peer_mirrors || rank < 0 || rank >= chain->world) return set_status(MLI_ERR_INVALID_ARG);
  uint64_t* ptrs[chain::kMaxPeers] = {};
  for (int r = 0; r < chain->world; ++r) {
    ptrs[r] = r == rank ? static_cast<uint64_t*>(chain->mirror_mem) : static_cast<uint64_t*>(peer_mirrors[r]);
    if (!ptrs[r]) return set_status(MLI_ERR_INVALID_ARG);
  }
  int cur = -1;
  cudaError_t err = cudaGetDevice(&cur);
  if (err == cudaSuccess && cur != chain->device) return set_status(MLI_ERR_INVALID_ARG);
  if (err == cudaSuccess)
    err = cudaMemcpy(const_cast<uint64_t**>(chain->args.peers), ptrs, sizeof(ptrs), cudaMemcpyHostToDevice);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  chain->args.world = chain->world;
  chain->peers_ready = true;
  return set_status(MLI_OK);
}

int mli_chain_rows(mli_chain* chain, int op, float* out, int* complete) {
  if (!chain || !out || !complete || op < 0 || op >= static_cast<int>(chain->ops.size()))
    return set_status(MLI_ERR_INVALID_ARG);
  const chain::Op& o = chain->ops[op];
  if (o.mirror < 0) return set_status(MLI_ERR_INVALID_ARG);
  unsigned seq = 0;
  cudaError_t err = cudaMemcpy(&seq, chain->args.seq, sizeof(seq), cudaMemcpyDeviceToHost);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  const unsigned last = seq == 1 ? chain::kSeqPeriod : seq - 1;  // the launch that ran last
  const size_t off = ((last & 1u) ? chain->args.mirror_half : 0u) + static_cast<size_t>(o.mirror);
  std::vector<uint64_t> w(static_cast<size_t>(o.d_total));
  err = cudaMemcpy(w.data(), chain->args.mirror + off, sizeof(uint64_t) * w.size(), cudaMemcpyDeviceToHost);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  const uint32_t tag = chain::row_tag(last, op);
  int ok = 1;
  for (size_t i = 0; i < w.size(); ++i) {
    ok &= static_cast<uint32_t>(w[i] >> 32) == tag;
    const uint32_t bits = static_cast<uint32_t>(w[i]);
    std::memcpy(out + i, &bits, sizeof(bits));
  }
  *complete = ok;
  return set_status(MLI_OK);
}

int mli_chain_run(mli_chain* chain, void* stream) {
  if (!chain || !chain->peers_ready) return set_status(MLI_ERR_INVALID_ARG);
  int cur = -1;
  cudaError_t err = cudaGetDevice(&cur);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  if (cur != chain->device) return set_status(MLI_ERR_INVALID_ARG);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(chain->grid);
  cfg.blockDim = dim3(chain->threads);
  cfg.dynamicSmemBytes = chain->smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, chain->kernel, chain->args));
}

int mli_chain_destroy(mli_chain* chain) {
  if (!chain) return set_status(MLI_ERR_INVALID_ARG);
  cudaError_t err = cudaFree(chain->dev_mem);
  const cudaError_t err2 = cudaFree(chain->mirror_mem);
  if (err == cudaSuccess) err = err2;
  delete chain;
  return err == cudaSuccess ? set_status(MLI_OK) : set_status(MLI_ERR_CUDA, err);
}

int mli_debug_plan_chain(const mli_gemv_op* ops, int count, int sm_count, int smem_optin,
                         int* out) {
  if (!out) return set_status(MLI_ERR_INVALID_ARG);
  chain::Plan p;
  const int rc = chain::plan_chain(ops, count, sm_count, smem_optin + 1024, smem_optin, 0u, nullptr, nullptr, &p);
  if (rc != MLI_OK) return set_status(rc);
  out[0] = p.grid;
  out[1] = static_cast<int>(p.smem);
  out[2] = p.args.ring;
  out[3] = static_cast<int>(p.args.slot_bytes);
  out[4] = p.args.units;
  out[5] = p.epochs;
  out[6] = p.args.n_phases;
  return set_status(MLI_OK);
}

}  // extern "C"
