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
//     64-column group is two K=32 MMAs into one of two int32 accumulators
//     (the second MMA accumulates onto the first), committed to an mbarrier;
//   * warps 2-9 are the epilogue: each reads its 32 accumulator rows over half
//     of the BN token columns (tcgen05.ld), converts the exact int32 group dot
//     and adds ws[r][g] * I into fp32 registers, then frees the accumulator.
// Tiles of K are split over CTAs so a layer fills the GPU; the last CTA of a
// tile sums the splits' partials in split order (deterministic) from the
// caller's workspace, scales by xs[t] and writes Y.
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
constexpr int kThreads = 320;        // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kEpiWarps = 8;
constexpr int kMaxAccBufs = 8;

// Accumulator buffers per tile width: as many as tensor memory holds (512
// columns), at most 8, so the MMAs run up to that many groups ahead of the
// epilogue.
__host__ __device__ constexpr int acc_bufs(int bn) { return 512 / bn < kMaxAccBufs ? 512 / bn : kMaxAccBufs; }

struct Args {
  float* y;
  const float* xs;
  const float* ws;
  float* partial;        // [splits][m][d] fp32 (splits > 1)
  unsigned* counters;    // [tiles] zero on entry and on exit (splits > 1)
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
};

__host__ __device__ constexpr uint32_t stage_bytes(int bn) { return 16384u + static_cast<uint32_t>(bn) * 128u; }
__host__ __device__ constexpr uint32_t smem_bytes(int bn) {
  return 1024u /* alignment slack */ + kStages * stage_bytes(bn) + 512u;
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
  return s;
}
__device__ __forceinline__ unsigned char* stage_a(const Smem& s, int i) { return s.ring + i * s.stage; }
__device__ __forceinline__ unsigned char* stage_b(const Smem& s, int i) { return s.ring + i * s.stage + 16384; }

__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
}

template <int kBN>
__global__ void __launch_bounds__(kThreads, 1)
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
          if (gi >= kAccBufs &&
              !mbar_wait_bounded(&sm.acc_empty[buf], ((gi / kAccBufs) - 1) & 1, kWaitLimitNs)) {
            ok = false;
            break;
          }
          tmem_fence_after();
          const uint32_t d = tmem + static_cast<uint32_t>(buf * kBN);
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            const uint32_t koff = static_cast<uint32_t>((2 * g + kk) * 32);
            mma_i8(d, sw128_desc(a_base + koff), sw128_desc(b_base + koff), idesc, kk > 0);
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
    griddep_wait();  // xs and the outputs belong to the stream order
    const int quad = warp & 3;                 // TMEM lanes 32*quad .. +31
    const int half = (warp - 2) >> 2;          // token columns [half*kBN/2, +kBN/2)
    constexpr int kCols = kBN / 2;
    const int row = row0 + 32 * quad + lane;
    const bool row_ok = row < a.d;
    float acc[kCols];
#pragma unroll
    for (int j = 0; j < kCols; ++j) acc[j] = 0.f;
    const float* ws_row = a.ws + static_cast<size_t>(row_ok ? row : 0) * a.G;
    bool ok = true;
    for (int gi = 0; gi < ngroups; ++gi) {
      const int buf = gi % kAccBufs;
      const int g = 2 * c_begin + gi;
      const float wsc = row_ok ? __ldg(ws_row + g) : 0.f;
      if (!mbar_wait_bounded(&sm.acc_full[buf], (gi / kAccBufs) & 1, kWaitLimitNs)) {
        ok = false;
        break;
      }
      tmem_fence_after();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * quad) << 16) +
                             static_cast<uint32_t>(buf * kBN + half * kCols);
      if constexpr (kCols >= 32) {
        uint32_t r[kCols / 32][32];
#pragma unroll
        for (int q = 0; q < kCols / 32; ++q) tmem_ld32(taddr + 32 * q, r[q]);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < kCols / 32; ++q)
#pragma unroll
          for (int j = 0; j < 32; ++j)
            acc[32 * q + j] = fmaf(static_cast<float>(static_cast<int>(r[q][j])), wsc, acc[32 * q + j]);
      } else {
        uint32_t r[kCols / 8][8];
#pragma unroll
        for (int q = 0; q < kCols / 8; ++q) tmem_ld8(taddr + 8 * q, r[q]);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < kCols / 8; ++q)
#pragma unroll
          for (int j = 0; j < 8; ++j)
            acc[8 * q + j] = fmaf(static_cast<float>(static_cast<int>(r[q][j])), wsc, acc[8 * q + j]);
      }
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
    }
    if (!ok) {
      record_device_error(kDevMmaTimeout);
      *sm.flag = 1;
    }
    epi_sync();
    const bool good = *sm.flag == 0;
    const int t_base = tok0 + half * kCols;
    if (good && a.splits == 1) {
      if (row_ok) {
#pragma unroll
        for (int j = 0; j < kCols; ++j) {
          const int t = t_base + j;
          if (t < a.m) a.y[static_cast<size_t>(t) * a.d + row] = acc[j] * a.xs[t];
        }
      }
    } else if (good) {
      // write this split's partial, then the last split of the tile reduces
      float* my_part = a.partial + static_cast<size_t>(split) * a.m * a.d;
      if (row_ok) {
#pragma unroll
        for (int j = 0; j < kCols; ++j) {
          const int t = t_base + j;
          if (t < a.m) my_part[static_cast<size_t>(t) * a.d + row] = acc[j];
        }
      }
      __threadfence();
      epi_sync();
      if (threadIdx.x == 64) {
        const unsigned prev = atomicAdd(a.counters + tile, 1u);
        *sm.flag = (prev == static_cast<unsigned>(a.splits - 1)) ? 2 : 0;
        if (prev == static_cast<unsigned>(a.splits - 1)) a.counters[tile] = 0;  // self-reset
        __threadfence();
      }
      epi_sync();
      if (*sm.flag == 2 && row_ok) {
        // Sum the splits in split order.  The split loop is outermost so the
        // loads of all columns of one split are independent and in flight
        // together.
        __threadfence();
        float v[kCols];
#pragma unroll
        for (int j = 0; j < kCols; ++j) v[j] = 0.f;
        for (int s2 = 0; s2 < a.splits; ++s2) {
          if (s2 == split) {
#pragma unroll
            for (int j = 0; j < kCols; ++j) v[j] += acc[j];
          } else {
            const float* src = a.partial + static_cast<size_t>(s2) * a.m * a.d + row;
            float pv[kCols];
#pragma unroll
            for (int j = 0; j < kCols; ++j) {
              const int t = t_base + j < a.m ? t_base + j : a.m - 1;
              pv[j] = __ldcg(src + static_cast<size_t>(t) * a.d);
            }
#pragma unroll
            for (int j = 0; j < kCols; ++j) v[j] += pv[j];
          }
        }
#pragma unroll
        for (int j = 0; j < kCols; ++j) {
          const int t = t_base + j;
          if (t < a.m) a.y[static_cast<size_t>(t) * a.d + row] = v[j] * a.xs[t];
        }
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
  return launch(gemm_w8a8_tc_kernel<kBN>, dim3(grid), dim3(kThreads), smem, stream, true, mw, mx, a);
}

}  // namespace tc

size_t gemm_tc_workspace_bytes(int m, int n, int d, int sm_count) {
  const tc::Plan p = tc::plan(m, n, d, sm_count, true);
  if (p.splits <= 1) return 256;
  return 256 + static_cast<size_t>(p.tiles_m) * p.tiles_n * sizeof(unsigned) +
         static_cast<size_t>(p.splits) * m * d * sizeof(float) + 256;
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
  if (p.splits > 1) {
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    a.counters = reinterpret_cast<unsigned*>(ws);
    const size_t cbytes = (static_cast<size_t>(p.tiles_m) * p.tiles_n * sizeof(unsigned) + 255) & ~size_t(255);
    a.partial = reinterpret_cast<float*>(ws + cbytes);
  }
  const int grid = p.tiles_m * p.tiles_n * p.splits;
  switch (p.bn) {
    case 16: err = tc::launch_bn<16>(mw, mx, a, grid, stream); break;
    case 32: err = tc::launch_bn<32>(mw, mx, a, grid, stream); break;
    case 64: err = tc::launch_bn<64>(mw, mx, a, grid, stream); break;
    default: err = tc::launch_bn<128>(mw, mx, a, grid, stream); break;
  }
  return check_cuda(err);
}

}  // namespace mli

// ---------------------------------------------------------------------------
// Allocation-free batched W8A8 (mli_gemm_w8a8_noalloc)
// ---------------------------------------------------------------------------
// Some callers cannot allocate device memory for a workspace: a plugin whose
// host framework owns every byte of device memory through its own pool, or a
// serving loop whose policy forbids allocations on the request path.  This
// entry point gives them the split-K tensor-core path anyway, with its scratch
// (the per-tile counters and the per-split partial sums) in a fixed array
// compiled into the library.  Every GPU that loads the library holds the array
// until the process exits.  The array is sized for the largest split-K
// workspace a B200 (148 SMs) can need: split-K never runs more partial tiles
// than there are SMs, and a partial tile is at most 128 rows x 128 tokens of
// fp32 (64 KiB), so 148 x 64 KiB plus the counters fits in 12 MiB.
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
  // The array keeps the previous call's contents: the tile counters must
  // start at zero, the partial sums are always written before they are read.
  const tc::Plan p = tc::plan(m, n, d, info.sm_count, true);
  if (p.splits > 1) {
    const size_t cbytes = static_cast<size_t>(p.tiles_m) * p.tiles_n * sizeof(unsigned);
    err = cudaMemsetAsync(g_noalloc_ptr[dev], 0, cbytes, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  }
  return gemm_w8a8_tc(y, xq, xs, w_q, w_s, m, n, d, g_noalloc_ptr[dev], kNoAllocWorkspaceBytes,
                      static_cast<cudaStream_t>(stream));
}
