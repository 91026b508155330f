// gemm_tc.cu -- batched W8A8 group-64 linear op on the B200 tensor cores
// (tcgen05.mma kind::i8, accumulators in tensor memory).
//
//   Y[t][r] = xs[t] * sum_g ws[r][g] * I[t][r][g],   I = exact int32 dot of
//   group g (64 columns) of weight row r with token t's int8 activation.
//
// The reference decodes one token at a time (src/model_cuda_v2_shared.cu:
// 465-501); with m >= 16 tokens the op is a real dense contraction and runs
// here.  One CTA computes a tile of 128 weight rows x BN tokens over a range of
// K:
//   * warp 0 streams 128-byte K chunks of the weight tile (128 x 128 B) and of
//     the activations (BN x 128 B) with 2-D TMA loads (128-byte swizzle, the
//     canonical K-major UMMA layout) into a 6-stage shared-memory ring;
//   * warp 1 owns the tensor memory and issues the MMAs from one thread: a
//     64-column group is two K=32 MMAs accumulating into one of up to eight
//     int32 accumulators, committed to an mbarrier;
//   * warps 2.. are the epilogue (4 lane quarters x up to 4 token-column
//     slices): each reads its 32 accumulator rows over its slice of the BN
//     token columns (tcgen05.ld), recovers the exact int32 group dot
//     as a float (the accumulators start at a bias that makes the int32 result
//     the bits of 1.5 * 2^23 + I), adds ws[r][g] * I into fp32 registers, and
//     refills the accumulator with the bias for its next use.
// Tiles of K are split over CTAs so a layer fills the GPU; each split writes
// its partial into the caller's workspace and a small kernel launched right
// after sums the splits in split order (deterministic) over the whole GPU,
// scales by xs[t] and writes Y.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "mli_common.cuh"
#include "mli_internal.h"

namespace mli {

namespace tc {

constexpr int kBM = 128;             // weight rows per tile (UMMA M)
constexpr int kChunk = 128;          // K bytes per stage (one 128-byte swizzle atom)
constexpr int kStages = 6;
// Warp 0 TMA, warp 1 MMA, warps 2.. epilogue: 4 lane quarters x kSlices token
// column slices (kCols columns each).  Two slices (8 epilogue warps): a
// measured tie with four, at more registers per thread and no spills.
template <int kBN>
struct Shape {
  static constexpr int kSlices = 2;
  static constexpr int kEpiWarps = 4 * kSlices;
  static constexpr int kThreads = (kEpiWarps + 2) * 32;
  static constexpr int kCols = kBN / kSlices;
};
constexpr int kMaxAccBufs = 8;

// Accumulator buffers per tile width: as many as tensor memory holds (512
// columns), at most 8, so the MMAs run up to that many groups ahead of the
// epilogue.
__host__ __device__ constexpr int acc_bufs(int bn) { return 512 / bn < kMaxAccBufs ? 512 / bn : kMaxAccBufs; }

struct Args {
  float* y;
  const float* xs;
  const float* ws;
  float* partial;        // [splits][m][d] fp32 (splits > 1): summed by splitk_reduce_kernel
  int m, n, d, G;
  int bn;                // tokens per tile (multiple of 16, <= 128)
  int tiles_m, tiles_n, splits, chunks;
};

// ---------------------------------------------------------------------------
// PTX wrappers (tcgen05, TMA tensor loads)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// K-major operand in the 128-byte-swizzle canonical layout: 8-row atoms of
// 128 bytes, atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t desc = 0;
  desc |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);        // start address
  desc |= static_cast<uint64_t>(1u) << 16;                       // leading offset (unused)
  desc |= static_cast<uint64_t>((1024u >> 4) & 0x3FFFu) << 32;   // stride offset: 8 rows
  desc |= static_cast<uint64_t>(1u) << 46;                       // descriptor version
  desc |= static_cast<uint64_t>(2u) << 61;                       // 128-byte swizzle
  return desc;
}

// kind::i8 instruction descriptor: s32 accumulate, signed int8 A and B, both
// K-major, M = 128, N = bn.
__device__ __forceinline__ uint32_t i8_idesc(int bn) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(bn >> 3) << 17) |
         (static_cast<uint32_t>(kBM >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(static_cast<uint32_t>(accumulate)), "r"(0u), "r"(0u),
      "r"(0u), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Accumulator bias: int32 accumulation onto the bits of 1.5 * 2^23 leaves the
// bits of the float 1.5 * 2^23 + I for any |I| < 2^22 (a group dot is at most
// 64 * 128 * 128 = 2^20 in magnitude), so one subtraction recovers (float)I
// exactly -- no int->float conversion instruction in the epilogue.
constexpr uint32_t kAccBias = 0x4B400000u;
constexpr float kAccBiasF = 12582912.0f;  // 1.5 * 2^23

// Fills this warp's 32 lanes x (8 * kN) columns at taddr with the bias.
template <int kN>
__device__ __forceinline__ void tmem_fill_bias(uint32_t taddr) {
  const uint32_t b = kAccBias;
#pragma unroll
  for (int q = 0; q < kN; ++q)
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(
                     taddr + 8 * q),
                 "r"(b), "r"(b), "r"(b), "r"(b), "r"(b), "r"(b), "r"(b), "r"(b)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 4-byte global -> shared asynchronous copy (no register round trip).
__device__ __forceinline__ void cp_async4(void* dst_smem, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Shared memory: ring of (A 16 KB | B bn*128 B) stages, 1024-byte aligned,
// then the barriers.
// ---------------------------------------------------------------------------
struct Smem {
  unsigned char* ring;   // stage s: A at ring + s * stage_bytes, B 16 KB after it
  uint32_t stage;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* acc_full;
  uint64_t* acc_empty;
  uint32_t* tmem_base;
  int* flag;
  float* ws;             // [kBM][kWsStride] group scales of the current window
  float* xs;             // [bn] activation scales of the tile's tokens
};

// The epilogue stages the tile's group scales ws[row][g] for a window of up to
// kWsWin groups in shared memory (row stride kWsStride floats, odd, so the
// 32 rows a warp reads at once fall in 32 banks): one burst of coalesced
// loads instead of a dependent global load per group.
constexpr int kWsWin = 48;
constexpr int kWsStride = kWsWin + 1;
constexpr uint32_t kWsBytes = kBM * kWsStride * 4u;

__host__ __device__ constexpr uint32_t stage_bytes(int bn) { return 16384u + static_cast<uint32_t>(bn) * 128u; }
__host__ __device__ constexpr uint32_t smem_bytes(int bn) {
  return 1024u /* alignment slack */ + kStages * stage_bytes(bn) + 512u + kWsBytes + 512u /* xs */;
}

__device__ __forceinline__ Smem carve(unsigned char* raw, int bn) {
  Smem s;
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(raw) + 1023u) & ~static_cast<uintptr_t>(1023u));
  s.ring = base;
  s.stage = stage_bytes(bn);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + kStages * stage_bytes(bn));
  s.full = bars;
  s.empty = bars + kStages;
  s.acc_full = bars + 2 * kStages;
  s.acc_empty = bars + 2 * kStages + kMaxAccBufs;
  s.tmem_base = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 2 * kMaxAccBufs);
  s.flag = reinterpret_cast<int*>(s.tmem_base + 1);
  s.ws = reinterpret_cast<float*>(base + kStages * stage_bytes(bn) + 512u);
  s.xs = s.ws + kBM * kWsStride;
  return s;
}
__device__ __forceinline__ unsigned char* stage_a(const Smem& s, int i) { return s.ring + i * s.stage; }
__device__ __forceinline__ unsigned char* stage_b(const Smem& s, int i) { return s.ring + i * s.stage + 16384; }

template <int kEpiWarps>
__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
}

template <int kBN>
__global__ void __launch_bounds__(Shape<kBN>::kThreads, 1)
    gemm_w8a8_tc_kernel(const __grid_constant__ CUtensorMap map_w,
                        const __grid_constant__ CUtensorMap map_x, const Args a) {
  extern __shared__ unsigned char smem_raw[];
  Smem sm = carve(smem_raw, kBN);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // tile / split of this CTA
  const int split = blockIdx.x % a.splits;
  const int tile = blockIdx.x / a.splits;
  const int tile_n = tile % a.tiles_n;
  const int tile_m = tile / a.tiles_n;
  const int row0 = tile_m * kBM;
  const int tok0 = tile_n * kBN;
  const int c_begin = static_cast<int>((static_cast<long long>(split) * a.chunks) / a.splits);
  const int c_end = static_cast<int>((static_cast<long long>(split + 1) * a.chunks) / a.splits);
  const int nchunks = c_end - c_begin;
  const int ngroups = 2 * nchunks;
  constexpr int kAccBufs = acc_bufs(kBN);
  constexpr int kEpiWarps = Shape<kBN>::kEpiWarps;
  constexpr uint32_t kTmemCols = kAccBufs * kBN;  // 128, 256 or 512: a power of two

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
    }
    for (int i = 0; i < kAccBufs; ++i) {
      mbar_init(&sm.acc_full[i], 1);
      mbar_init(&sm.acc_empty[i], kEpiWarps);
    }
    *sm.flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(sm.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = *sm.tmem_base;
  griddep_launch_dependents();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      // Weights never depend on the previous kernel: fill the ring's weight
      // halves first, then wait for the activations.
      const int first = nchunks < kStages ? nchunks : kStages;
      for (int c = 0; c < first; ++c) {
        mbar_arrive_expect_tx(&sm.full[c], stage_bytes(kBN));
        tma_load_2d(stage_a(sm, c), &map_w, (c_begin + c) * kChunk, row0, &sm.full[c]);
      }
      griddep_wait();
      for (int c = 0; c < first; ++c) tma_load_2d(stage_b(sm, c), &map_x, (c_begin + c) * kChunk, tok0, &sm.full[c]);
      for (int c = kStages; c < nchunks; ++c) {
        const int s = c % kStages;
        if (!mbar_wait_bounded(&sm.empty[s], ((c / kStages) - 1) & 1, kWaitLimitNs)) {
          record_device_error(kDevMmaTimeout);
          *sm.flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&sm.full[s], stage_bytes(kBN));
        const int kx = (c_begin + c) * kChunk;
        tma_load_2d(stage_a(sm, s), &map_w, kx, row0, &sm.full[s]);
        tma_load_2d(stage_b(sm, s), &map_x, kx, tok0, &sm.full[s]);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = i8_idesc(kBN);
      int gi = 0;
      bool ok = true;
      for (int c = 0; c < nchunks && ok; ++c) {
        const int s = c % kStages;
        if (!mbar_wait_bounded(&sm.full[s], (c / kStages) & 1, kWaitLimitNs)) {
          ok = false;
          break;
        }
        tmem_fence_after();
        const uint32_t a_base = smem_u32(stage_a(sm, s));
        const uint32_t b_base = smem_u32(stage_b(sm, s));
        for (int g = 0; g < 2; ++g, ++gi) {
          const int buf = gi % kAccBufs;
          // use u of a buffer waits for phase u: the epilogue's bias fill
          // (phase 0) or its read of use u - 1
          if (!mbar_wait_bounded(&sm.acc_empty[buf], (gi / kAccBufs) & 1, kWaitLimitNs)) {
            ok = false;
            break;
          }
          tmem_fence_after();
          const uint32_t d = tmem + static_cast<uint32_t>(buf * kBN);
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            const uint32_t koff = static_cast<uint32_t>((2 * g + kk) * 32);
            mma_i8(d, sw128_desc(a_base + koff), sw128_desc(b_base + koff), idesc, true);
          }
          mma_commit(&sm.acc_full[buf]);
        }
        mma_commit(&sm.empty[s]);  // the stage is free once its MMAs have read it
      }
      if (!ok) {
        record_device_error(kDevMmaTimeout);
        *sm.flag = 1;
      }
    }
  } else {
    // ---------------- epilogue (warps 2..9) ----------------
    const int quad = warp & 3;                 // TMEM lanes 32*quad .. +31
    const int half = (warp - 2) >> 2;          // token column slice [half*kCols, +kCols)
    constexpr int kCols = Shape<kBN>::kCols;
    const int row = row0 + 32 * quad + lane;
    const bool row_ok = row < a.d;
    float acc[kCols];
#pragma unroll
    for (int j = 0; j < kCols; ++j) acc[j] = 0.f;
    const int et = static_cast<int>(threadIdx.x) - 64;  // epilogue thread 0..255
    // every accumulator buffer starts at the bias
    const uint32_t tlane = tmem + (static_cast<uint32_t>(32 * quad) << 16) + static_cast<uint32_t>(half * kCols);
#pragma unroll
    for (int b = 0; b < kAccBufs; ++b) tmem_fill_bias<kCols / 8>(tlane + static_cast<uint32_t>(b * kBN));
    tmem_wait_st();
    tmem_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int b = 0; b < kAccBufs; ++b) mbar_arrive(&sm.acc_empty[b]);
    griddep_wait();  // xs and the outputs belong to the stream order
    bool ok = true;
    for (int gi = 0; gi < ngroups; ++gi) {
      const int buf = gi % kAccBufs;
      if (gi % kWsWin == 0) {
        // stage the scales of groups gi .. gi + wn - 1 of the tile's rows:
        // two threads per row, every copy in flight at once
        const int wn = ngroups - gi < kWsWin ? ngroups - gi : kWsWin;
        epi_sync<kEpiWarps>();  // every epilogue thread is done with the previous window
        constexpr int kTpr = kEpiWarps * 32 / kBM;  // threads per row
        const int rl = et / kTpr, rr = row0 + rl;
        float* dst = sm.ws + rl * kWsStride;
        if (rr < a.d) {
          const float* src = a.ws + static_cast<size_t>(rr) * a.G + 2 * c_begin + gi;
          for (int g = et % kTpr; g < wn; g += kTpr) cp_async4(dst + g, src + g);
        } else {
          for (int g = et % kTpr; g < wn; g += kTpr) dst[g] = 0.f;
        }
        if (gi == 0 && et < kBN) sm.xs[et] = tok0 + et < a.m ? __ldg(a.xs + tok0 + et) : 0.f;
        cp_async_wait_all();
        epi_sync<kEpiWarps>();
      }
      const float wsc = sm.ws[(32 * quad + lane) * kWsStride + gi % kWsWin];
      // After a timeout the warp keeps walking the groups without waiting, so
      // that every epilogue warp meets the same window barriers.
      if (ok && !mbar_wait_bounded(&sm.acc_full[buf], (gi / kAccBufs) & 1, kWaitLimitNs)) ok = false;
      if (!ok) continue;
      tmem_fence_after();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * quad) << 16) +
                             static_cast<uint32_t>(buf * kBN + half * kCols);
      if constexpr (kCols >= 32) {
        // 32 columns at a time: fewer live registers next to acc[kCols]
#pragma unroll
        for (int q = 0; q < kCols / 32; ++q) {
          uint32_t r[32];
          tmem_ld32(taddr + 32 * q, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            acc[32 * q + j] = fmaf(__uint_as_float(r[j]) - kAccBiasF, wsc, acc[32 * q + j]);
        }
        tmem_fill_bias<kCols / 8>(taddr);  // ready for the buffer's next use
      } else {
        uint32_t r[kCols / 8][8];
#pragma unroll
        for (int q = 0; q < kCols / 8; ++q) tmem_ld8(taddr + 8 * q, r[q]);
        tmem_wait_ld();
        tmem_fill_bias<kCols / 8>(taddr);
#pragma unroll
        for (int q = 0; q < kCols / 8; ++q)
#pragma unroll
          for (int j = 0; j < 8; ++j)
            acc[8 * q + j] = fmaf(__uint_as_float(r[q][j]) - kAccBiasF, wsc, acc[8 * q + j]);
      }
      tmem_wait_st();
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
    }
    if (!ok) {
      record_device_error(kDevMmaTimeout);
      *sm.flag = 1;
    }
    epi_sync<kEpiWarps>();
    const bool good = *sm.flag == 0;
    const int t_base = tok0 + half * kCols;
    if (good && a.splits == 1) {
      if (row_ok) {
#pragma unroll
        for (int j = 0; j < kCols; ++j) {
          const int t = t_base + j;
          if (t < a.m) a.y[static_cast<size_t>(t) * a.d + row] = acc[j] * sm.xs[half * kCols + j];
        }
      }
    } else if (good && row_ok) {
      // this split's partial; splitk_reduce_kernel sums the splits in order
      float* my_part = a.partial + static_cast<size_t>(split) * a.m * a.d;
#pragma unroll
      for (int j = 0; j < kCols; ++j) {
        const int t = t_base + j;
        if (t < a.m) my_part[static_cast<size_t>(t) * a.d + row] = acc[j];
      }
    }
  }

  // Tensor memory is released by its owner warp once every role is done.
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                 : "memory");
  }
}

// Split-K: y[t][r] = xs[t] * sum_s partial[s][t][r], the splits summed in split
// order (deterministic), over the whole GPU at once.  Launched right after
// the GEMM (programmatic dependent launch): the partials are read only after
// griddepcontrol.wait.
constexpr int kReduceThreads = 256;
constexpr int kReduceElems = 4;  // consecutive outputs per thread

__global__ void __launch_bounds__(kReduceThreads)
    splitk_reduce_kernel(float* y, const float* partial, const float* xs, int splits, int m, int d) {
  griddep_wait();
  const size_t md = static_cast<size_t>(m) * d;
  const size_t i0 = (static_cast<size_t>(blockIdx.x) * kReduceThreads + threadIdx.x) * kReduceElems;
  if (i0 >= md) return;
  float v[kReduceElems];
#pragma unroll
  for (int e = 0; e < kReduceElems; ++e) v[e] = 0.f;
  int s = 0;
  for (; s + 4 <= splits; s += 4) {  // four splits' loads in flight
    float p[4][kReduceElems];
#pragma unroll
    for (int b = 0; b < 4; ++b)
#pragma unroll
      for (int e = 0; e < kReduceElems; ++e)
        p[b][e] = i0 + e < md ? __ldcg(partial + static_cast<size_t>(s + b) * md + i0 + e) : 0.f;
#pragma unroll
    for (int b = 0; b < 4; ++b)
#pragma unroll
      for (int e = 0; e < kReduceElems; ++e) v[e] += p[b][e];
  }
  for (; s < splits; ++s)
#pragma unroll
    for (int e = 0; e < kReduceElems; ++e)
      v[e] += i0 + e < md ? __ldcg(partial + static_cast<size_t>(s) * md + i0 + e) : 0.f;
#pragma unroll
  for (int e = 0; e < kReduceElems; ++e) {
    const size_t i = i0 + e;
    if (i < md) y[i] = v[e] * __ldg(xs + i / d);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D int8 map over [rows][cols] row-major, box 128 bytes x box_rows, 128-byte
// swizzle (the canonical K-major UMMA layout); rows past the end read zero.
bool make_map(CUtensorMap* map, const void* base, int rows, int cols, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kChunk), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct Plan {
  int bn, tiles_m, tiles_n, splits, chunks;
};

Plan plan(int m, int n, int d, int sm_count, bool have_ws) {
  Plan p;
  p.bn = m <= 16 ? 16 : (m <= 32 ? 32 : (m <= 64 ? 64 : 128));
  p.tiles_m = (d + kBM - 1) / kBM;
  p.tiles_n = (m + p.bn - 1) / p.bn;
  p.chunks = n / kChunk;
  // Split K so the tiles fill the SMs in one wave, keeping at least two
  // 128-byte chunks (four groups) per split.
  const int tiles = p.tiles_m * p.tiles_n;
  int splits = have_ws ? sm_count / tiles : 1;
  if (splits > p.chunks / 2) splits = p.chunks / 2;
  if (splits < 1) splits = 1;
  p.splits = splits;
  return p;
}

template <int kBN>
cudaError_t launch_bn(const CUtensorMap& mw, const CUtensorMap& mx, const Args& a, int grid,
                      cudaStream_t stream) {
  const uint32_t smem = smem_bytes(kBN);
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(gemm_w8a8_tc_kernel<kBN>), smem);
  if (e != cudaSuccess) return e;
  return launch(gemm_w8a8_tc_kernel<kBN>, dim3(grid), dim3(Shape<kBN>::kThreads), smem, stream, true, mw, mx, a);
}

}  // namespace tc

size_t gemm_tc_workspace_bytes(int m, int n, int d, int sm_count) {
  const tc::Plan p = tc::plan(m, n, d, sm_count, true);
  if (p.splits <= 1) return 256;
  return 256 + static_cast<size_t>(p.splits) * m * d * sizeof(float);
}

// Tensor-core path: m >= 16, n % 128 == 0, group 64, 16-byte aligned
// operands.  Returns MLI_ERR_UNSUPPORTED (without launching) otherwise.
int gemm_w8a8_tc(float* y, const int8_t* xq, const float* xs, const int8_t* w_q, const float* w_s,
                 int m, int n, int d, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (m < 16 || n % tc::kChunk != 0 || !aligned(xq, 16) || !aligned(w_q, 16))
    return MLI_ERR_UNSUPPORTED;
  cudaError_t err = cudaSuccess;
  const DeviceInfo& dev = current_device(&err);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  const bool have_ws = workspace != nullptr &&
                       workspace_bytes >= gemm_tc_workspace_bytes(m, n, d, dev.sm_count);
  const tc::Plan p = tc::plan(m, n, d, dev.sm_count, have_ws);
  CUtensorMap mw, mx;
  if (!tc::make_map(&mw, w_q, d, n, tc::kBM) || !tc::make_map(&mx, xq, m, n, p.bn))
    return MLI_ERR_UNSUPPORTED;
  tc::Args a = {};
  a.y = y;
  a.xs = xs;
  a.ws = w_s;
  a.m = m;
  a.n = n;
  a.d = d;
  a.G = n / 64;
  a.bn = p.bn;
  a.tiles_m = p.tiles_m;
  a.tiles_n = p.tiles_n;
  a.splits = p.splits;
  a.chunks = p.chunks;
  if (p.splits > 1) a.partial = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + 256);
  const int grid = p.tiles_m * p.tiles_n * p.splits;
  switch (p.bn) {
    case 16: err = tc::launch_bn<16>(mw, mx, a, grid, stream); break;
    case 32: err = tc::launch_bn<32>(mw, mx, a, grid, stream); break;
    case 64: err = tc::launch_bn<64>(mw, mx, a, grid, stream); break;
    default: err = tc::launch_bn<128>(mw, mx, a, grid, stream); break;
  }
  if (err != cudaSuccess || p.splits == 1) return check_cuda(err);
  const size_t per_block = static_cast<size_t>(tc::kReduceThreads) * tc::kReduceElems;
  const size_t md = static_cast<size_t>(m) * d;
  const unsigned blocks = static_cast<unsigned>((md + per_block - 1) / per_block);
  return check_cuda(launch(tc::splitk_reduce_kernel, dim3(blocks), dim3(tc::kReduceThreads), 0, stream, true,
                           y, static_cast<const float*>(a.partial), xs, p.splits, m, d));
}

}  // namespace mli

// ---------------------------------------------------------------------------
// Allocation-free batched W8A8 (mli_gemm_w8a8_noalloc)
// ---------------------------------------------------------------------------
// Some callers cannot allocate device memory for a workspace: a plugin whose
// host framework owns every byte of device memory through its own pool, or a
// serving loop whose policy forbids allocations on the request path.  This
// entry point gives them the split-K tensor-core path anyway, with its scratch
// (the per-split partial sums) in a fixed array
// compiled into the library.  Every GPU that loads the library holds the array
// until the process exits.  The array is sized for the largest split-K
// workspace a B200 (148 SMs) can need: split-K never runs more partial tiles
// than there are SMs, and a partial tile is at most 128 rows x 128 tokens of
// fp32 (64 KiB), so 148 x 64 KiB fits in 12 MiB.
namespace mli {
namespace {

constexpr size_t kNoAllocWorkspaceBytes = 12u << 20;
static __device__ __align__(256) unsigned char g_noalloc_workspace[kNoAllocWorkspaceBytes];

constexpr int kMaxDevicesNoAlloc = 64;
std::once_flag g_noalloc_once[kMaxDevicesNoAlloc];
void* g_noalloc_ptr[kMaxDevicesNoAlloc];
cudaError_t g_noalloc_err[kMaxDevicesNoAlloc];

}  // namespace
}  // namespace mli

extern "C" int mli_gemm_w8a8_noalloc(float* y, const int8_t* xq, const float* xs,
                                     const int8_t* w_q, const float* w_s, int m, int n, int d,
                                     int group_size, void* stream) {
  using namespace mli;
  if (!y || !xq || !xs || !w_q || !w_s || m <= 0 || n <= 0 || d <= 0 || group_size <= 0)
    return set_status(MLI_ERR_INVALID_ARG);
  // Only the tensor-core shapes use scratch; everything else is rejected
  // rather than silently run elsewhere.
  if (group_size != 64 || m < 16 || n % tc::kChunk != 0 || !aligned(xq, 16) || !aligned(w_q, 16))
    return set_status(MLI_ERR_UNSUPPORTED);
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  if (dev < 0 || dev >= kMaxDevicesNoAlloc) return set_status(MLI_ERR_UNSUPPORTED);
  // Once per device, with that device current: the array's device address.
  // In host code g_noalloc_workspace only names a host-side stand-in, so the
  // kernel must be given this address, never the symbol itself.
  std::call_once(g_noalloc_once[dev], [dev]() {
    g_noalloc_err[dev] = cudaGetSymbolAddress(&g_noalloc_ptr[dev], g_noalloc_workspace);
  });
  if (g_noalloc_err[dev] != cudaSuccess) return set_status(MLI_ERR_CUDA, g_noalloc_err[dev]);
  const DeviceInfo& info = current_device(&err);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  const size_t need = gemm_tc_workspace_bytes(m, n, d, info.sm_count);
  if (need > kNoAllocWorkspaceBytes) return set_status(MLI_ERR_UNSUPPORTED);
  // The array keeps the previous call's contents; nothing in it needs to
  // start at zero (the partial sums are always written before they are read).
  return gemm_w8a8_tc(y, xq, xs, w_q, w_s, m, n, d, g_noalloc_ptr[dev], kNoAllocWorkspaceBytes,
                      static_cast<cudaStream_t>(stream));
}
