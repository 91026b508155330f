// gemv_g64.cu -- batch-1 INT8 group-64 GEMV for B200 (sm_100a).
//
// Two forms of the reference's linear op (src/model_cuda_v2_shared.cu):
//   W8A32  y[r] = sum_c (q[r][c] * s[r][c/64]) * x[c]        (:36-62)
//   W8A8   y[r] = sum_g ((float)I[r][g] * s[r][g]) * xs     (:465-501)
//          I[r][g] = exact int32 dot of group g of row r with the int8 x.
//
// The op is HBM-bound (one weight byte per two flops), so the kernel is built
// to keep HBM streaming across the whole chain of GEMVs of a decode step:
//
//  * Bulk-copy streaming.  "Stages" of whole weight rows (and their scale
//    rows) move from HBM into a ring of shared-memory slots with 1-D bulk
//    copies (the TMA engine, completion on an mbarrier); eight warps compute
//    from shared memory.  A stage is ~32 KB of contiguous int8 rows, the ring
//    holds 2-6 stages per CTA.  Whichever warp is last to finish with a slot
//    refills it, so no warp ever waits for another to drain a slot.
//  * Programmatic dependent launch.  Every CTA triggers its dependents as it
//    starts and fills its ring *before* griddepcontrol.wait (weights never
//    depend on the previous kernel).  One CTA per SM uses half of the SM's
//    registers and at most half of its shared memory, so the next GEMV's CTA
//    is resident alongside and fills its ring while this one drains.
//  * Consumers: warp w owns one slice of a row -- 1024 columns for W8A32,
//    2048 for W8A8 (split-K when n is wider) -- and takes 4 (W8A32) or 2
//    (W8A8) rows of it per stage, reduced across lanes together.  In read k
//    of a row, lane l takes the 16 bytes at 16*(l + 32k) of its slice, so a
//    warp read is 512 contiguous bytes (conflict-free), and the slice of x it
//    needs is the same for every row: it lives in registers for the whole
//    kernel.
//  * The activation is read only after griddepcontrol.wait, straight from
//    global memory (it was just written, so it sits in L2), and prepared once
//    per CTA in shared memory:
//      W8A32: split exactly enough for fp32 parity into two int16 planes of
//      digit pairs under a per-group power of two (see x_digits_prologue), so
//      every weight chunk is 16 dp2a of exact int32 sums plus a few fp32 ops
//      instead of 16 int8->fp32 conversions and 16 FMAs;
//      W8A8 fused: quantised in the prologue, bit-identical to
//      quantize_activation.
//  * W8A8 does four dp4a per 16 bytes, a 3-shuffle quad reduce-scatter that
//    leaves each lane with one whole group's int32 dot, then the reference's
//    per-group term ((float)I * ws) * xs.
//  * Slices of one row are combined in slice order by the last consumer warp
//    to finish the stage.  A row's arithmetic depends only on n: never on d,
//    the stage, the grid or the GPU count, so a row-sharded classifier gives
//    bit-identical logits on any number of GPUs.
#include <utility>

#include "gemv_rows.cuh"
#include "mli_common.cuh"
#include "mli_internal.h"

namespace mli {

constexpr int kThreads = kConsumerThreads;
constexpr int kMaxSlices = 8;
constexpr int kMaxRing = 6;
constexpr int kHeader = 256;

// Shared-memory header: full[6] @0, reduction scratch (8 floats) @128,
// per-slot completion counters (6 ints) @160, reduction indices (8 ints)
// @192, CTA flags @224.
struct Smem {
  uint64_t* full;
  float* red;
  int* counters;
  int* red_i;
  int* broken;
  __device__ explicit Smem(unsigned char* base)
      : full(reinterpret_cast<uint64_t*>(base)),
        red(reinterpret_cast<float*>(base + 128)),
        counters(reinterpret_cast<int*>(base + 160)),
        red_i(reinterpret_cast<int*>(base + 192)),
        broken(reinterpret_cast<int*>(base + 224)) {}
};

struct StreamArgs {
  float* y;
  const float* x;   // fp32 activation (W8A32, fused W8A8)
  const int8_t* xq; // int8 activation (W8A8)
  const float* xs;  // activation scale (W8A8)
  int8_t* xq_out;   // fused W8A8: optional copy of the quantised x ...
  float* xs_out;    // ... and of its scale
  const int8_t* w;
  const float* s;
  int n, d, G;      // G = n / 64 groups per row
  int S, wps;       // slices per row, consumer warps per slice (8 / S)
  int R;            // rows per stage
  int n_stages;     // ceil(d / R)
  int ring;         // ring slots
  uint32_t stage_bytes;  // R * n + R * G * 4
  uint32_t x_off, ring_off, part_off;
  // Row-sharded output (world > 0): row r of this launch is global row
  // row_offset + r; its value is stored, tagged with the step, into every
  // rank's logits words peer_y[p] ([2][d_total], the half chosen by
  // *step & 1), and every CTA stores its rows' (max, first index) as one
  // tagged partial word into every rank's block (no counters, no fences).
  int world, rank, row_offset, d_total;
  uint32_t out_off;  // shared-memory staging of this CTA's output rows
  const unsigned* step;
  unsigned long long* peer_y[kMaxPeers];
  // Fused argmax (row-sharded, out != nullptr): the last CTA of the launch
  // polls every rank's partial words of this step, reduces them to the
  // argmax, writes it and advances the step.
  long long* out;
  unsigned* step_rw;                   // this rank's step counter
  unsigned* ctas_done;                 // this rank's finished-CTA count (zero between launches)
  unsigned long long timeout_ns;
  int shard_ctas[kMaxPeers];
};

// ---------------------------------------------------------------------------
// The streaming kernel
// ---------------------------------------------------------------------------
// Stores one finished output row: locally, or (row-sharded) into the CTA's
// shared staging; row-sharded launches publish a CTA's rows (a contiguous
// range) to every rank as one coalesced burst at the end of the CTA, which
// costs less than per-stage remote stores.
template <bool kPeer>
__device__ __forceinline__ void store_row(const StreamArgs& a, int row, float v, float* staged,
                                          int cta_row0) {
  if constexpr (!kPeer) {
    a.y[row] = v;
  } else {
    staged[row - cta_row0] = v;
  }
}

// (max, first index) over v[0..n) by the CTA's 256 threads, scanning each
// thread's elements in index order with a strict `>` and combining with the
// first-maximum rule (larger value, then smaller index).  Result on thread 0.
__device__ __forceinline__ void cta_first_max(const float* v, int n, int idx0, float* red_v,
                                              int* red_i, float* out_v, int* out_i) {
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < n; i += kConsumerThreads)
    if (v[i] > bv) { bv = v[i]; bi = idx0 + i; }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  if ((threadIdx.x & 31) == 0) {
    red_v[threadIdx.x >> 5] = bv;
    red_i[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kConsumerWarps; ++w)
      if (red_v[w] > bv || (red_v[w] == bv && red_i[w] < bi)) { bv = red_v[w]; bi = red_i[w]; }
    *out_v = bv;
    *out_i = bi;
  }
}

// Issues the bulk copies of stage `st` (rows st*R .. +R-1 and their scales)
// into ring slot `slot`, completing on full[slot].
__device__ __forceinline__ void issue_stage(const StreamArgs& a, unsigned char* ring, uint64_t* full,
                                            int st, int slot) {
  const int row0 = st * a.R;
  const int rows = min(a.R, a.d - row0);
  const uint32_t wb = static_cast<uint32_t>(rows) * a.n;
  const uint32_t sb = static_cast<uint32_t>(rows) * a.G * 4u;
  unsigned char* dst = ring + static_cast<size_t>(slot) * a.stage_bytes;
  mbar_arrive_expect_tx(&full[slot], wb + sb);
  bulk_copy_g2s(dst, a.w + static_cast<size_t>(row0) * a.n, wb, &full[slot]);
  bulk_copy_g2s(dst + static_cast<size_t>(a.R) * a.n, a.s + static_cast<size_t>(row0) * a.G, sb,
                &full[slot]);
}

template <Form F, bool kPeer>
__global__ void __launch_bounds__(kThreads, 2) gemv_stream_kernel(const StreamArgs a) {
  extern __shared__ __align__(1024) unsigned char smem[];
  Smem sm(smem);
  unsigned char* ring = smem + a.ring_off;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long T = a.n_stages;
  const int begin = static_cast<int>((blockIdx.x * T) / gridDim.x);
  const int cnt = static_cast<int>(((blockIdx.x + 1) * T) / gridDim.x) - begin;

  // Fill the ring before waiting on the previous kernel: weights never
  // depend on it.
  if (threadIdx.x == 0) {
    for (int i = 0; i < a.ring; ++i) {
      mbar_init(&sm.full[i], 1);
      sm.counters[i] = 0;
    }
    *sm.broken = 0;
    fence_barrier_init();
    for (int i = 0; i < a.ring && i < cnt; ++i) issue_stage(a, ring, sm.full, begin + i, i);
  }
  __syncthreads();
  griddep_launch_dependents();

  constexpr int K = chunks_per_lane(F);
  constexpr int kSlice = slice_cols(F);
  constexpr int RB = rows_per_warp(F);
  const int S = a.S;
  const int sl = warp % S, wj = warp / S;
  const bool warp_on = wj < a.wps;
  const int g_slice = min(8 * K, a.G - sl * 8 * K);
  unsigned vmask = 0;
#pragma unroll
  for (int k = 0; k < K; ++k)
    if (warp_on && (lane >> 2) + 8 * k < g_slice) vmask |= 1u << k;
  const int col0 = sl * kSlice + 16 * lane;  // first column of this lane's chunk 0

  // The activation is the previous kernel's output: read it only now.
  griddep_wait();
  const unsigned parity = kPeer ? (*a.step & 1u) : 0u;
  float* staged = reinterpret_cast<float*>(smem + a.out_off);
  const int cta_row0 = begin * a.R;
  float xscale = 0.f;
  uint4 xd[2][4];  // W8A32 digit pairs of chunks 0, 1 (load_digit_chunk)
  float fac[2];
  uint4 xv[4];     // W8A8 int8 chunks 0..3
  if constexpr (F == Form::kW8A32) {
    int8_t* planes = reinterpret_cast<int8_t*>(smem + a.x_off);
    float* facs = reinterpret_cast<float*>(planes + 4 * a.n);
    x_digits_prologue(a.x, a.n, planes, facs);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const bool v = (vmask >> k) & 1u;
      if (v) {
        load_digit_chunk(planes, a.n, col0 + 512 * k, xd[k]);
      } else {
#pragma unroll
        for (int p = 0; p < 4; ++p) xd[k][p] = make_uint4(0, 0, 0, 0);
      }
      fac[k] = v ? facs[(col0 + 512 * k) >> 6] : 0.f;
    }
  } else if constexpr (F == Form::kW8A8Fused) {
    int8_t* q8 = reinterpret_cast<int8_t*>(smem + a.x_off);
    xscale = x_quant_prologue(a.x, a.n, q8, sm.red);
    __syncthreads();
    if (blockIdx.x == 0) {
      if (a.xq_out != nullptr) {
        if ((reinterpret_cast<uintptr_t>(a.xq_out) & 15) == 0) {
          for (int i = threadIdx.x * 16; i < a.n; i += kConsumerThreads * 16)
            *reinterpret_cast<uint4*>(a.xq_out + i) = *reinterpret_cast<const uint4*>(q8 + i);
        } else {
          for (int i = threadIdx.x; i < a.n; i += kConsumerThreads) a.xq_out[i] = q8[i];
        }
      }
      if (a.xs_out != nullptr && threadIdx.x == 0) *a.xs_out = xscale;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k)
      xv[k] = ((vmask >> k) & 1u) ? *reinterpret_cast<const uint4*>(q8 + col0 + 512 * k)
                                  : make_uint4(0, 0, 0, 0);
  } else {
    xscale = *a.xs;
#pragma unroll
    for (int k = 0; k < 4; ++k)
      xv[k] = ((vmask >> k) & 1u) ? *reinterpret_cast<const uint4*>(a.xq + col0 + 512 * k)
                                  : make_uint4(0, 0, 0, 0);
  }

  if constexpr (kPeer) __syncthreads();  // x region becomes the output staging area

  for (int i = 0; i < cnt; ++i) {
    const int slot = i % a.ring;
    if (!mbar_wait_bounded(&sm.full[slot], (i / a.ring) & 1, kWaitLimitNs)) {
      record_device_error(kDevStageTimeout);
      *sm.broken = 1;
      // give a copy still in flight the same time to land, then leave
      mbar_wait_bounded(&sm.full[slot], (i / a.ring) & 1, kWaitLimitNs);
      break;
    }
    const int row0 = (begin + i) * a.R;
    const int rows = min(a.R, a.d - row0);
    const int8_t* wst = reinterpret_cast<const int8_t*>(ring + static_cast<size_t>(slot) * a.stage_bytes);
    const float* sst = reinterpret_cast<const float*>(wst + static_cast<size_t>(a.R) * a.n);
    float* part = reinterpret_cast<float*>(smem + a.part_off) + slot * a.R * S;
    if (warp_on) {
      const int j0 = wj * RB;  // this warp's rows of the stage: j0 .. j0 + RB - 1
      const int nvalid = rows - j0;
      if (nvalid > 0) {
        const int8_t* wr = wst + static_cast<size_t>(j0) * a.n + sl * kSlice;
        const float* sr = sst + j0 * a.G + sl * 8 * K;
        float v[RB];
        if constexpr (F == Form::kW8A32)
          rows_w8a32<RB>(wr, sr, a.n, a.G, nvalid, xd, fac, vmask, lane, v);
        else
          rows_w8a8<RB>(wr, sr, a.n, a.G, nvalid, xv, vmask, lane, xscale, v);
        const float total = warp_sum_rows<RB>(v, lane);
        constexpr int kLanesPerRow = 32 / RB;
        const int r = lane / kLanesPerRow;
        if ((lane & (kLanesPerRow - 1)) == 0 && r < nvalid) {
          if (S == 1) store_row<kPeer>(a, row0 + j0 + r, total, staged, cta_row0);
          else part[(j0 + r) * S + sl] = total;
        }
      }
    }
    // The last warp to finish with this slot sums the slices of its rows and
    // refills the slot with stage i + ring.
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      __threadfence_block();
      last = atomicAdd(&sm.counters[slot], 1) == kConsumerWarps - 1;
      if (last) sm.counters[slot] = 0;
      __threadfence_block();
    }
    if (__shfl_sync(0xffffffffu, last, 0)) {
      if (S > 1) {
        for (int rr = lane; rr < rows; rr += 32) {
          float v = part[rr * S];
          for (int s2 = 1; s2 < S; ++s2) v += part[rr * S + s2];
          store_row<kPeer>(a, row0 + rr, v, staged, cta_row0);
        }
      }
      if (lane == 0 && i + a.ring < cnt) {
        fence_proxy_async_smem();  // this CTA's reads of the slot precede the copy's writes
        issue_stage(a, ring, sm.full, begin + i + a.ring, slot);
      }
      __syncwarp();
    }
  }
  if constexpr (kPeer) {
    // Publish the CTA's rows to every rank as one coalesced burst of tagged
    // words, then the rows' (max, first index) as one tagged partial word per
    // rank.  A reader knows a word has arrived by its tag, so nothing here
    // waits for a fence.  A CTA that gave up on a stage publishes nothing.
    __syncthreads();
    const bool broken = *sm.broken != 0;
    const unsigned tag = rowshard_tag(*a.step);
    if (!broken) {
      const int cta_rows = max(0, min((begin + cnt) * a.R, a.d) - cta_row0);
      __shared__ float s_best_v;
      __shared__ int s_best_i;
      cta_first_max(staged, cta_rows, a.row_offset + cta_row0, sm.red, sm.red_i, &s_best_v, &s_best_i);
      __syncthreads();
      const size_t off = static_cast<size_t>(parity) * a.d_total + a.row_offset + cta_row0;
      for (int p = 0; p < a.world; ++p) {
        unsigned long long* dst = a.peer_y[p] + off;
        for (int i = threadIdx.x; i < cta_rows; i += kConsumerThreads)
          st_relaxed_sys_b64(dst + i, tag_word(__float_as_uint(staged[i]), tag));
        if (threadIdx.x == 0 && cta_rows > 0) {
          unsigned long long* slot = rowshard_partials(a.peer_y[p], a.d_total) +
                                     (static_cast<size_t>(parity) * kMaxPeers + a.rank) * kMaxRankCtas + blockIdx.x;
          st_relaxed_sys_b64(slot, tag_word(__float_as_uint(s_best_v),
                                            (static_cast<unsigned>(s_best_i) << 12) | tag));
        }
      }
    }
    if (a.out == nullptr) return;
    // Fused argmax: the last CTA to finish takes over (every other CTA of
    // the launch has stored its words by then).
    __shared__ int s_last;
    if (threadIdx.x == 0) s_last = atomicAdd(a.ctas_done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    if (threadIdx.x == 0) *a.ctas_done = 0;  // every other CTA of this launch is done with it
    __shared__ int s_int;
    const unsigned s = *a.step;
    const long long best =
        rowshard_poll_argmax<kConsumerThreads>(a.peer_y[a.rank], a.d_total, s & 1u, rowshard_tag(s), a.world,
                                               a.shard_ctas, a.timeout_ns, sm.red, sm.red_i, &s_int);
    if (threadIdx.x == 0) {
      if (best < 0) record_device_error(kDevPeerTimeout);
      *a.out = best;
      if (best >= 0) *a.step_rw = s + 1;
    }
  }
}

// ---------------------------------------------------------------------------
// Generic kernels: any group size, any n, any alignment.  One warp per row,
// byte loads; the reference's semantics (columns past (n / gs) * gs are
// ignored, as its groups_per_row = n / group_size truncates).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    gemv_w8a32_generic_kernel(float* y, const float* x, const int8_t* w,
                              const float* s, int n, int d, int gs) {
  griddep_wait();
  const int row = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= d) return;
  const int ng = n / gs;
  const int8_t* wr = w + static_cast<size_t>(row) * n;
  const float* sr = s + static_cast<size_t>(row) * ng;
  float acc = 0.f;
  for (int g = 0; g < ng; ++g) {
    float part = 0.f;
    for (int j = lane; j < gs; j += 32)
      part = fmaf(static_cast<float>(wr[g * gs + j]), x[g * gs + j], part);
    acc = fmaf(part, sr[g], acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) y[row] = acc;
}

__global__ void __launch_bounds__(256)
    gemv_w8a8_generic_kernel(float* y, const int8_t* xq, const float* xs,
                             const int8_t* w, const float* s, int n, int d,
                             int gs) {
  griddep_wait();
  const int row = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= d) return;
  const int ng = n / gs;
  const int8_t* wr = w + static_cast<size_t>(row) * n;
  const float* sr = s + static_cast<size_t>(row) * ng;
  const float xscale = *xs;
  float acc = 0.f;
  for (int g = 0; g < ng; ++g) {
    int part = 0;
    for (int j = lane; j < gs; j += 32)
      part += static_cast<int>(wr[g * gs + j]) * static_cast<int>(xq[g * gs + j]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
    acc += (static_cast<float>(part) * sr[g]) * xscale;
  }
  if (lane == 0) y[row] = acc;
}

__global__ void __launch_bounds__(256)
    group_dots_kernel(int32_t* out, const int8_t* xq, const int8_t* w, int n,
                      int d, int gs) {
  const int ng = n / gs;
  const size_t total = static_cast<size_t>(d) * ng;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t row = i / ng;
    const int g = static_cast<int>(i - row * ng);
    const int8_t* wr = w + row * n + static_cast<size_t>(g) * gs;
    const int8_t* xr = xq + static_cast<size_t>(g) * gs;
    int acc = 0;
    for (int j = 0; j < gs; ++j) acc += static_cast<int>(wr[j]) * static_cast<int>(xr[j]);
    out[i] = acc;
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Stage geometry and shared-memory layout.  Returns false if the shape does
// not fit the streaming kernel.
bool plan_stream(Form f, const DeviceInfo& dev, int n, int d, bool peer, StreamArgs* a,
                 size_t* smem_out, int* grid_out) {
  a->n = n;
  a->d = d;
  a->G = n / kGroup;
  a->S = (n + slice_cols(f) - 1) / slice_cols(f);
  if (a->S > kMaxSlices) return false;
  a->wps = kConsumerWarps / a->S;
  const int R = rows_per_warp(f) * a->wps;
  a->R = R;
  a->n_stages = (d + R - 1) / R;
  a->stage_bytes = static_cast<uint32_t>(R) * n + static_cast<uint32_t>(R) * a->G * 4u;
  // W8A32: two digit-pair planes + per-group factors; fused W8A8: the int8 x.
  size_t xbytes =
      (f == Form::kW8A32) ? 4u * n + (n / kGroup) * 4u : (f == Form::kW8A8 ? 0u : static_cast<size_t>(n));
  // Row-sharded launches stage a CTA's output rows (at most
  // ceil(stages / min(stages, SMs)) stages of R rows) in the same region.
  if (peer) {
    const int g1 = a->n_stages < dev.sm_count ? a->n_stages : dev.sm_count;
    const size_t out_bytes = static_cast<size_t>((a->n_stages + g1 - 1) / g1) * R * 4u;
    if (out_bytes > 64 * 1024) return false;
    if (out_bytes > xbytes) xbytes = out_bytes;
  }
  a->x_off = kHeader;
  a->ring_off = static_cast<uint32_t>(align_up(kHeader + xbytes, 128));
  const size_t part_bytes = a->S > 1 ? static_cast<size_t>(R) * a->S * 4u : 0;

  // Half of the SM's shared memory (minus the per-CTA reservation) lets the
  // next kernel's CTA co-reside; fall back to a whole SM for huge rows.
  const size_t half = static_cast<size_t>(dev.smem_per_sm) / 2 - 1024;
  const size_t whole = static_cast<size_t>(dev.smem_optin_per_cta);
  int ring = 0;
  for (size_t budget : {half, whole}) {
    if (budget <= a->ring_off) continue;
    ring = static_cast<int>((budget - a->ring_off) / (a->stage_bytes + part_bytes + 16));
    if (ring >= 2) break;
  }
  if (ring < 2) return false;
  if (ring > kMaxRing) ring = kMaxRing;
  a->ring = ring;
  a->part_off = static_cast<uint32_t>(align_up(a->ring_off + static_cast<size_t>(ring) * a->stage_bytes, 16));
  // Output rows are staged where the activation was prepared: every warp has
  // copied its slice of x into registers before the first row is stored.
  a->out_off = a->x_off;
  *smem_out = a->part_off + ring * part_bytes;
  // Two CTAs per SM (16 warps computing) once the matrix has two stages per
  // SM; smaller ones take one slot and leave the second to the next kernel in
  // the stream, which then fills its ring while this one runs.
  const int min_stages_two = (launch_flags() & MLI_LAUNCH_ONE_CTA) ? 16 : 2;
  const int per_sm = (a->n_stages >= min_stages_two * dev.sm_count &&
                      2 * (*smem_out + 1024) <= static_cast<size_t>(dev.smem_per_sm)) ? 2 : 1;
  *grid_out = a->n_stages < per_sm * dev.sm_count ? a->n_stages : per_sm * dev.sm_count;
  return true;
}

bool fast_path_ok(int n, int group_size) { return group_size == kGroup && n % 256 == 0; }

// Launches the streaming kernel; returns MLI_ERR_UNSUPPORTED (without
// launching) when the shape does not fit, so the caller can fall back.
int launch_stream(Form f, StreamArgs args, int n, int d, cudaStream_t stream) {
  cudaError_t err = cudaSuccess;
  const DeviceInfo& dev = current_device(&err);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  size_t smem = 0;
  int grid = 0;
  if (!plan_stream(f, dev, n, d, args.world > 0, &args, &smem, &grid)) return MLI_ERR_UNSUPPORTED;
  if (args.world > 0 && grid > kMaxRankCtas) return set_status(MLI_ERR_UNSUPPORTED);
  const bool peer = args.world > 0;
  void (*kfn)(const StreamArgs) = nullptr;
  switch (f) {
    case Form::kW8A32:
      kfn = peer ? gemv_stream_kernel<Form::kW8A32, true> : gemv_stream_kernel<Form::kW8A32, false>;
      break;
    case Form::kW8A8:
      kfn = peer ? gemv_stream_kernel<Form::kW8A8, true> : gemv_stream_kernel<Form::kW8A8, false>;
      break;
    case Form::kW8A8Fused:
      kfn = peer ? gemv_stream_kernel<Form::kW8A8Fused, true> : gemv_stream_kernel<Form::kW8A8Fused, false>;
      break;
  }
  err = ensure_dynamic_smem(reinterpret_cast<const void*>(kfn), smem);
  if (err != cudaSuccess) return check_cuda(err);
  err = launch(kfn, dim3(grid), dim3(kThreads), smem, stream, true, args);
  return check_cuda(err);
}

}  // namespace

// Grid of the row-sharded streaming GEMV for `rows` rows of width n on the
// current device (0 if the launch would not fit), for the waiting side.
int rowshard_grid(int form, int n, int rows) {
  if (rows <= 0) return 0;
  cudaError_t err = cudaSuccess;
  const DeviceInfo& dev = current_device(&err);
  if (err != cudaSuccess) return -1;
  StreamArgs a = {};
  size_t smem = 0;
  int grid = 0;
  if (!plan_stream(form == 0 ? Form::kW8A32 : Form::kW8A8Fused, dev, n, rows, true, &a, &smem, &grid))
    return -1;
  return grid;
}

namespace {

dim3 warp_per_row_grid(int d) { return dim3(static_cast<unsigned>((d + 7) / 8)); }

}  // namespace

// Launches the quantiser of m tokens (quant.cu).
int launch_quantize_rows(int8_t* xq, float* xs, const float* x, int m, int n,
                         cudaStream_t stream);

}  // namespace mli

using namespace mli;

extern "C" {

int mli_gemv_w8a32(float* y, const float* x, const int8_t* w_q, const float* w_s,
                   int n, int d, int group_size, void* stream) {
  if (!y || !x || !w_q || !w_s || n <= 0 || d <= 0 || group_size <= 0)
    return set_status(MLI_ERR_INVALID_ARG);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (fast_path_ok(n, group_size) && aligned(x, 16) && aligned(w_q, 16) && aligned(w_s, 16)) {
    StreamArgs a = {};
    a.y = y; a.x = x; a.w = w_q; a.s = w_s;
    const int rc = launch_stream(Form::kW8A32, a, n, d, st);
    if (rc != MLI_ERR_UNSUPPORTED) return rc;
  }
  return check_cuda(launch(gemv_w8a32_generic_kernel, warp_per_row_grid(d), dim3(256), 0, st,
                           true, y, x, w_q, w_s, n, d, group_size));
}

int mli_gemv_w8a8(float* y, const int8_t* xq, const float* xs, const int8_t* w_q,
                  const float* w_s, int n, int d, int group_size, void* stream) {
  if (!y || !xq || !xs || !w_q || !w_s || n <= 0 || d <= 0 || group_size <= 0)
    return set_status(MLI_ERR_INVALID_ARG);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (fast_path_ok(n, group_size) && aligned(xq, 16) && aligned(w_q, 16) && aligned(w_s, 16)) {
    StreamArgs a = {};
    a.y = y; a.xq = xq; a.xs = xs; a.w = w_q; a.s = w_s;
    const int rc = launch_stream(Form::kW8A8, a, n, d, st);
    if (rc != MLI_ERR_UNSUPPORTED) return rc;
  }
  return check_cuda(launch(gemv_w8a8_generic_kernel, warp_per_row_grid(d), dim3(256), 0, st,
                           true, y, xq, xs, w_q, w_s, n, d, group_size));
}

int mli_gemv_w8a8_fused(float* y, int8_t* xq_out, float* xs_out, const float* x,
                        const int8_t* w_q, const float* w_s, int n, int d,
                        int group_size, void* stream) {
  if (!y || !x || !w_q || !w_s || n <= 0 || d <= 0 || group_size <= 0)
    return set_status(MLI_ERR_INVALID_ARG);
  if ((xq_out == nullptr) != (xs_out == nullptr)) return set_status(MLI_ERR_INVALID_ARG);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (fast_path_ok(n, group_size) && aligned(x, 16) && aligned(w_q, 16) && aligned(w_s, 16)) {
    StreamArgs a = {};
    a.y = y; a.x = x; a.xq_out = xq_out; a.xs_out = xs_out; a.w = w_q; a.s = w_s;
    const int rc = launch_stream(Form::kW8A8Fused, a, n, d, st);
    if (rc != MLI_ERR_UNSUPPORTED) return rc;
  }
  // Unfused path for shapes outside the streaming kernel: needs caller buffers.
  if (xq_out == nullptr) return set_status(MLI_ERR_UNSUPPORTED);
  int rc = launch_quantize_rows(xq_out, xs_out, x, 1, n, st);
  if (rc != MLI_OK) return rc;
  return mli_gemv_w8a8(y, xq_out, xs_out, w_q, w_s, n, d, group_size, stream);
}

int mli_gemv_rowshard(int form, unsigned long long* const* peer_logits, const unsigned* step,
                      const float* x, const int8_t* w_q, const float* w_s, int n, int rows, int row_offset,
                      int d_total, int rank, int world, int group_size, void* stream) {
  if (!peer_logits || !step || !x || world <= 0 || world > kMaxPeers || rank < 0 || rank >= world ||
      rows < 0 || row_offset < 0 || row_offset + rows > d_total || n <= 0 || group_size <= 0 ||
      (form != 0 && form != 2))
    return set_status(MLI_ERR_INVALID_ARG);
  for (int p = 0; p < world; ++p)
    if (!peer_logits[p]) return set_status(MLI_ERR_INVALID_ARG);
  if (d_total >= kMaxRowshardRows) return set_status(MLI_ERR_UNSUPPORTED);
  if (rows == 0) return set_status(MLI_OK);
  if (!w_q || !w_s) return set_status(MLI_ERR_INVALID_ARG);
  if (!fast_path_ok(n, group_size) || !aligned(x, 16) || !aligned(w_q, 16) || !aligned(w_s, 16))
    return set_status(MLI_ERR_UNSUPPORTED);
  StreamArgs a = {};
  a.x = x; a.w = w_q; a.s = w_s;
  a.world = world; a.rank = rank; a.row_offset = row_offset; a.d_total = d_total; a.step = step;
  for (int p = 0; p < world; ++p) a.peer_y[p] = peer_logits[p];
  return launch_stream(form == 0 ? Form::kW8A32 : Form::kW8A8Fused, a, n, rows,
                       static_cast<cudaStream_t>(stream));
}

int mli_gemv_rowshard_argmax(int form, unsigned long long* const* peer_logits, void* own_block,
                             const float* x, const int8_t* w_q, const float* w_s, int n,
                             int rows, int row_offset, int d_total, int rank, int world,
                             int group_size, const int* shard_rows, long long* out,
                             int timeout_us, void* stream) {
  if (!peer_logits || !own_block || !x || !shard_rows || !out || world <= 0 ||
      world > kMaxPeers || rank < 0 || rank >= world || rows <= 0 || row_offset < 0 ||
      row_offset + rows > d_total || n <= 0 || group_size <= 0 || timeout_us <= 0 ||
      (form != 0 && form != 2) || !w_q || !w_s)
    return set_status(MLI_ERR_INVALID_ARG);
  for (int p = 0; p < world; ++p)
    if (!peer_logits[p]) return set_status(MLI_ERR_INVALID_ARG);
  if (d_total >= kMaxRowshardRows) return set_status(MLI_ERR_UNSUPPORTED);
  if (!fast_path_ok(n, group_size) || !aligned(x, 16) || !aligned(w_q, 16) || !aligned(w_s, 16))
    return set_status(MLI_ERR_UNSUPPORTED);
  StreamArgs a = {};
  a.x = x; a.w = w_q; a.s = w_s;
  a.world = world; a.rank = rank; a.row_offset = row_offset; a.d_total = d_total;
  unsigned char* blk = static_cast<unsigned char*>(own_block);
  a.step = reinterpret_cast<const unsigned*>(blk + 128);
  a.step_rw = reinterpret_cast<unsigned*>(blk + 128);
  a.ctas_done = reinterpret_cast<unsigned*>(blk + 192);
  a.out = out;
  a.timeout_ns = static_cast<unsigned long long>(timeout_us) * 1000ull;
  long long total = 0;
  const Form f = form == 0 ? Form::kW8A32 : Form::kW8A8Fused;
  for (int p = 0; p < world; ++p) {
    a.peer_y[p] = peer_logits[p];
    if (shard_rows[p] <= 0) return set_status(MLI_ERR_INVALID_ARG);
    a.shard_ctas[p] = rowshard_grid(form, n, shard_rows[p]);
    if (a.shard_ctas[p] <= 0 || a.shard_ctas[p] > kMaxRankCtas) return set_status(MLI_ERR_UNSUPPORTED);
    total += shard_rows[p];
  }
  if (total != d_total || shard_rows[rank] != rows) return set_status(MLI_ERR_INVALID_ARG);
  return launch_stream(f, a, n, rows, static_cast<cudaStream_t>(stream));
}

int mli_debug_plan_gemv(int form, int n, int d, int sm_count, int smem_per_sm,
                        int smem_optin, int* out) {
  if (!out || form < 0 || form > 2 || n <= 0 || d <= 0 || sm_count <= 0 || smem_per_sm <= 0 ||
      smem_optin <= 0)
    return set_status(MLI_ERR_INVALID_ARG);
  if (!fast_path_ok(n, kGroup)) return set_status(MLI_ERR_UNSUPPORTED);
  DeviceInfo dev;
  dev.sm_count = sm_count;
  dev.smem_per_sm = smem_per_sm;
  dev.smem_optin_per_cta = smem_optin;
  StreamArgs a = {};
  size_t smem = 0;
  int grid = 0;
  if (!plan_stream(static_cast<Form>(form), dev, n, d, false, &a, &smem, &grid))
    return set_status(MLI_ERR_UNSUPPORTED);
  out[0] = grid;
  out[1] = static_cast<int>(smem);
  out[2] = a.S;
  out[3] = a.wps;
  out[4] = a.R;
  out[5] = a.n_stages;
  out[6] = a.ring;
  out[7] = static_cast<int>(a.stage_bytes);
  return set_status(MLI_OK);
}

int mli_debug_group_dots(int32_t* out, const int8_t* xq, const int8_t* w_q, int n,
                         int d, int group_size, void* stream) {
  if (!out || !xq || !w_q || n <= 0 || d <= 0 || group_size <= 0)
    return set_status(MLI_ERR_INVALID_ARG);
  const size_t total = static_cast<size_t>(d) * (n / group_size);
  const size_t want = (total + 255) / 256;
  const unsigned blocks = static_cast<unsigned>(want < 65535 ? (want > 0 ? want : 1) : 65535);
  return check_cuda(launch(group_dots_kernel, dim3(blocks), dim3(256), 0,
                           static_cast<cudaStream_t>(stream), false, out, xq, w_q, n, d,
                           group_size));
}

}  // extern "C"
