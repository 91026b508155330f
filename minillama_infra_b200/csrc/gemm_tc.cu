// gemm_tc.cu -- batched W8A8 group-64 linear op on the B200 tensor cores
// (tcgen05.mma kind::i8, accumulators in tensor memory).
//
//   Y[t][r] = xs[t] * sum_g ws[r][g] * I[t][r][g],   I = exact int32 dot of
//   group g (64 columns) of weight row r with token t's int8 activation.
//
// The reference decodes one token at a time (src/model_cuda_v2_shared.cu:
// 465-501); with m >= 16 tokens the op is a real dense contraction and runs
// here, in one of two kernels chosen per call:
//
// Split-K tiles (gemm_w8a8_tc_kernel<BN>, BN = 16..128 tokens).  One CTA
// computes a tile of 128 weight rows x BN tokens over a range of K:
//   * warp 0 streams 128-byte K chunks of the weight tile (128 x 128 B) and
//     of the activation tile (BN x 128 B) with 2-D TMA loads (128-byte
//     swizzle, the canonical K-major UMMA layout) into a ring of 6-10 stages;
//   * warp 1 owns the tensor memory and issues the MMAs from one thread (two
//     threads, warps 1 and 2 on alternate chunks, for tiles of 32 tokens or
//     fewer): per 64-column group two K = 32 MMAs into an int32 accumulator
//     buffer (128-token tiles first write the accumulator offset with one
//     MMA of a constant unsigned tile), one commit per unit of buffers and
//     one for the stage;
//   * warpgroups 1 and 2 are the epilogue, taking alternate units: each warp
//     reads its 32 accumulator lanes over all BN token columns (tcgen05.ld),
//     recovers the exact int32 group dot as a float (the accumulator starts
//     at an offset that makes its bits a float linear in the dot), adds
//     ws[r][g] * I into fp32 registers (packed f32x2 arithmetic) and, for
//     narrow tiles, refills the offset with tensor-memory stores; the two
//     warpgroups' sums are added in a fixed order at the end.
//   K is split over CTAs so a layer fills the GPU.  The splits of a tile run
//   as one thread-block cluster: each stages its partial tile in shared memory
//   and sums a share of the tile over the cluster's partials in split order
//   (deterministic), scales by xs[t] and writes Y.  Where clusters of the
//   wanted size do not fit the GPU at once, the splits may instead write their
//   partials into the caller's workspace, summed in split order by a second,
//   GPU-wide kernel.
//
// Persistent whole tiles (gemm_w8a8_persistent_kernel, more than 64 tokens,
// problems with enough 128 x 128 tiles to keep every SM evenly busy): one CTA
// per SM walks a host-made list of whole tiles, its TMA, MMA and epilogue
// counters running on across tiles; the epilogue warpgroups split a tile by
// token columns and store complete rows straight to Y (described at the
// kernel).
//
// This file builds as a device module of its own (whole-program compilation,
// no -rdc): only then does ptxas allocate the epilogue's registers up to its
// setmaxnreg share.  Its kernels reach the library's device error word
// through a pointer.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#define MLI_SEPARATE_DEVICE_MODULE
#include "mli_common.cuh"
#include "mli_internal.h"

namespace mli {

namespace tc {

constexpr int kBM = 128;             // weight rows per tile (UMMA M); a token's tile row is 32 float4s
constexpr int kChunk = 128;          // K bytes per stage (one 128-byte swizzle atom)
constexpr int kStageA = kBM * kChunk;  // 16 KB of weights per stage
// A stage holds one 128-byte K chunk of the weight tile (16 KB) and of the
// activation tile (bn x 128 B); 192 KB of stages.
__host__ __device__ constexpr uint32_t stage_bytes(int bn) { return kStageA + static_cast<uint32_t>(bn) * kChunk; }
__host__ __device__ constexpr int stages(int bn) {
  return 196608u / stage_bytes(bn) < 12u ? static_cast<int>(196608u / stage_bytes(bn)) : 12;
}
constexpr int kMaxStages = 12;
// Warpgroup 0: warp 0 TMA, warp 1 MMA (warps 2 and 3 idle).  Warpgroups 1
// and 2 are the epilogue, ping-ponging over the K chunks (the two groups of
// chunk c go to warpgroup 1 + c % 2), so that one warpgroup's tensor-memory
// loads, refills and waits overlap the other's arithmetic.  Each epilogue warp covers every token column of the 32
// accumulator lanes of its rank in the warpgroup (warp % 4).
template <int kBN>
struct Shape {
  static constexpr int kEpiWarps = 8;
  static constexpr int kFirstEpiWarp = 4;
  static constexpr int kThreads = 12 * 32;
  static constexpr int kCols = kBN;
  static constexpr int kLdCols = 16;  // accumulator columns per tensor-memory load
  // wide tiles keep 128 fp32 sums per epilogue thread: registers move from
  // the producer warpgroup to the epilogue warpgroups
  static constexpr bool kSplitRegs = kBN >= 64;
  // 128-token tiles: the accumulator offset is written by one extra MMA per
  // group (a constant unsigned tile, see kMmaBias* below) instead of
  // tensor-memory stores from the epilogue, and every 64-column group is a
  // unit of its own, so that each epilogue warpgroup has two buffers (the
  // MMAs fill one while it reads the other).  Narrower tiles refill by
  // stores (one store of 16 columns per group) and hand over a chunk's two
  // groups as one unit.
  static constexpr bool kMmaBias = kBN >= 128;
  static constexpr int kUnitGroups = kMmaBias ? 1 : 2;
};
// Registers per thread after the setmaxnreg split: the producer warpgroup
// gives up what its loops do not need, the epilogue warpgroups take it (the
// fp32 sums of a whole lane row of the tile stay in registers).  The split
// must fit the registers the block is launched with; launch_bn checks that
// against the compiled kernel before the first launch.
constexpr int kRegsProducer = 88;
constexpr int kRegsEpilogue = 208;
constexpr int kRegsBlock = 128 * (kRegsProducer + 2 * kRegsEpilogue);
constexpr int kMaxAccBufs = 8;
constexpr int kMaxUnits = 4;  // 4 single-group units at 128 tokens, 4 chunk pairs of 8 buffers below

// Accumulator buffers per tile width: as many as tensor memory holds (512
// columns), at most 8, so the MMAs run up to that many groups ahead of the
// epilogue.
__host__ __device__ constexpr int acc_bufs(int bn) { return 512 / bn < kMaxAccBufs ? 512 / bn : kMaxAccBufs; }

struct Args {
  float* y;
  const float* xs;
  const float* ws;
  float* partial;        // [splits][m][d] fp32 (splits > 1, no cluster): summed by splitk_reduce_kernel
  int m, n, d, G;
  int bn;                // tokens per tile (multiple of 16, <= 128)
  int tiles_m, tiles_n, splits, chunks;
  int cluster;           // > 1: the splits of a tile form one cluster and sum over shared memory
  int vec4;              // outputs may be written as aligned float4 (d % 4 == 0, 16-byte aligned)
  unsigned int* err;     // the library's device error word
};

__device__ __forceinline__ void record_device_error(const Args& a, unsigned int code) {
  if (a.err) atomicCAS(a.err, 0u, code);
}

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
// The same with unsigned int8 A and B (the accumulator-offset MMA).
__device__ __forceinline__ uint32_t u8_idesc(int bn) {
  return (2u << 4) | (static_cast<uint32_t>(bn >> 3) << 17) | (static_cast<uint32_t>(kBM >> 4) << 24);
}
// K-major operand of one 32-byte K step in the 32-byte-swizzle layout: rows of
// 32 bytes, 8-row atoms of 256 bytes; 128 rows span 4 KB.
__device__ __forceinline__ uint64_t sw32_desc(uint32_t saddr) {
  uint64_t desc = 0;
  desc |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);       // start address
  desc |= static_cast<uint64_t>(1u) << 16;                      // leading offset (unused)
  desc |= static_cast<uint64_t>((256u >> 4) & 0x3FFFu) << 32;   // stride offset: 8 rows
  desc |= static_cast<uint64_t>(1u) << 46;                      // descriptor version
  desc |= static_cast<uint64_t>(6u) << 61;                      // 32-byte swizzle
  return desc;
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

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
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
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
// This warp's 32 lanes x kCols consecutive accumulator columns at taddr.
template <int kCols>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[kCols]) {
  if constexpr (kCols >= 32) {
#pragma unroll
    for (int q = 0; q < kCols / 32; ++q) tmem_ld32(taddr + 32 * q, r + 32 * q);
  } else if constexpr (kCols == 16) {
    tmem_ld16(taddr, r);
  } else {
    static_assert(kCols == 8, "8, 16 or a multiple of 32 columns");
    tmem_ld8(taddr, r);
  }
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// The same wait, tied to the 16 registers of the load it completes: their
// uses cannot be scheduled before it.
__device__ __forceinline__ void tmem_wait_ld16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                 "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

// Accumulator bias: int32 accumulation onto the bits of 1.5 * 2^23 leaves the
// bits of the float 1.5 * 2^23 + I for any |I| < 2^22 (a group dot is at most
// 64 * 128 * 128 = 2^20 in magnitude), so one subtraction recovers (float)I
// exactly -- no int->float conversion instruction in the epilogue.
constexpr uint32_t kAccBias = 0x4B400000u;
constexpr float kAccBiasF = 12582912.0f;  // 1.5 * 2^23

// Offset written by an MMA (128-token tiles).  One K = 32 step of unsigned
// int8 A = B = a constant tile whose every 16-byte chunk holds kMmaBiasChunk
// (bytes 255 x 8, 63, 10, 3, 3, 1, 0, 0, 0: squares summing to 2^19) leaves
// V0 = 2 * 2^19 = 2^20 in every accumulator, whatever the swizzle does to the
// chunks.  The group dot then leaves bits V0 + I, 0 < V0 + I < 2^23 for any
// int8 operands (|I| <= 2^20, I > -2^20), which read as a float are the
// subnormal (V0 + I) * 2^-149: one exact subtraction of 2^-129 gives
// I * 2^-149.  The group scale enters as ws * 2^90 (exact), so the fused
// multiply-add adds I * ws * 2^-59 with the rounding of I * ws, and the tile
// is scaled by 2^59 (exact) before it leaves the registers.  Exact for group
// scales in [2^-67, 2^38); a finite scale of 2^38 or more is refused through
// the error word.
constexpr uint32_t kMmaBiasBits = 1u << 20;        // the float 2^-129
constexpr uint32_t kMmaScaleIn = 0x6C800000u;      // 2^90
constexpr uint32_t kMmaScaleOut = 0x5D000000u;     // 2^59
constexpr uint32_t kBiasTileBytes = 4096;          // 128 rows x 32 bytes
__device__ __forceinline__ uint4 mma_bias_chunk() { return make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0x03030A3Fu, 0x1u); }

// Fills this warp's 32 lanes x kCols columns at taddr with the bias: a store's
// source is as many consecutive registers as it has columns, so 16 columns
// per store keep 16 registers of the bias live (8 at 8 columns).
template <int kCols>
__device__ __forceinline__ void tmem_fill_bias(uint32_t taddr) {
  const uint32_t b = kAccBias;
  if constexpr (kCols % 16 == 0) {
#pragma unroll
    for (int q = 0; q < kCols / 16; ++q)
      asm volatile(
          "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(
              taddr + 16 * q),
          "r"(b)
          : "memory");
  } else {
    static_assert(kCols == 8, "8 or a multiple of 16 columns");
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr), "r"(b)
                 : "memory");
  }
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Two fp32 lanes per instruction (sm_100 packed f32x2 arithmetic); each lane
// rounds exactly like the scalar instruction.
__device__ __forceinline__ uint64_t f2_pack(uint32_t lo, uint32_t hi) {
  uint64_t v;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "r"(lo), "r"(hi));
  return v;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
// acc + (biased - bias) * w, per lane: (float)I * ws accumulated as before.
__device__ __forceinline__ uint64_t f2_unbias_fma(uint64_t biased, uint64_t bias, uint64_t w, uint64_t acc) {
  uint64_t t, d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(t) : "l"(biased), "l"(bias));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(t), "l"(w), "l"(acc));
  return d;
}

// 4-byte global -> shared asynchronous copy (no register round trip).
__device__ __forceinline__ void cp_async4(void* dst_smem, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// Thread-block cluster barrier over every thread of every block of the
// cluster; release/acquire order the shared-memory writes before it with the
// reads of other blocks after it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\nbarrier.cluster.wait.acquire;" ::: "memory");
}
// Address of the same shared-memory location in block `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_peer(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ int ld_cluster_s32(uint32_t addr) {
  int v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

// Four consecutive outputs of token t, rows r .. r + 3 (those below d).
__device__ __forceinline__ void store_out4(float* dst, const Args& a, int t, int r, float4 v) {
  float* p = dst + static_cast<size_t>(t) * a.d + r;
  if (a.vec4 && r + 3 < a.d) {
    *reinterpret_cast<float4*>(p) = v;
  } else {
    const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (r + i < a.d) p[i] = e[i];
  }
}

// ---------------------------------------------------------------------------
// Shared memory (1024-byte aligned): the ring of stages,
// the barriers, the group-scale window and the token scales.
// ---------------------------------------------------------------------------
struct Smem {
  unsigned char* ring;   // stage i at ring + i * stage: weights, then activations
  uint32_t stage;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* acc_full;    // per unit of accumulator buffers
  uint64_t* acc_empty;
  unsigned char* bias;   // the offset MMA's constant operand (128-token tiles)
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
static_assert(kWsWin % 4 == 0, "a window holds whole chunk pairs of both epilogue warpgroups");
constexpr uint32_t kWsBytes = kBM * kWsStride * 4u;
constexpr uint32_t kBarBytes = 512u;

__host__ __device__ constexpr uint32_t rings_bytes(int bn) { return stages(bn) * stage_bytes(bn); }
__host__ __device__ constexpr uint32_t smem_bytes(int bn) {
  return 1024u /* alignment slack */ + rings_bytes(bn) + kBiasTileBytes + kBarBytes + kWsBytes + 512u /* xs */;
}
static_assert(smem_bytes(128) <= 232448 && smem_bytes(64) <= 232448 && smem_bytes(32) <= 232448 &&
                  smem_bytes(16) <= 232448,
              "shared memory per block");
static_assert((2 * kMaxStages + 2 * kMaxUnits) * 8 + 8 <= kBarBytes, "barrier area");
static_assert(stage_bytes(128) % 1024 == 0 && stage_bytes(64) % 1024 == 0 && stage_bytes(32) % 1024 == 0 &&
                  stage_bytes(16) % 1024 == 0,
              "the offset tile after the ring stays 1024-byte aligned");
// the finished tile ([bn][kBM] fp32) is staged in the ring
static_assert(128 * kBM * 4 <= rings_bytes(128) && 64 * kBM * 4 <= rings_bytes(64) &&
                  32 * kBM * 4 <= rings_bytes(32) && 16 * kBM * 4 <= rings_bytes(16),
              "output tile in the ring");

__device__ __forceinline__ Smem carve(unsigned char* raw, int bn) {
  Smem s;
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(raw) + 1023u) & ~static_cast<uintptr_t>(1023u));
  s.ring = base;
  s.stage = stage_bytes(bn);
  s.bias = base + rings_bytes(bn);  // 1024-byte aligned: every stage is a multiple of 1 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(s.bias + kBiasTileBytes);
  s.full = bars;
  s.empty = bars + kMaxStages;
  s.acc_full = bars + 2 * kMaxStages;
  s.acc_empty = bars + 2 * kMaxStages + kMaxUnits;
  s.tmem_base = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 2 * kMaxUnits);
  s.flag = reinterpret_cast<int*>(s.tmem_base + 1);
  s.ws = reinterpret_cast<float*>(s.bias + kBiasTileBytes + kBarBytes);
  s.xs = s.ws + kBM * kWsStride;
  return s;
}
__device__ __forceinline__ unsigned char* stage_a(const Smem& s, int i) { return s.ring + i * s.stage; }
__device__ __forceinline__ unsigned char* stage_b(const Smem& s, int i) { return s.ring + i * s.stage + kStageA; }

// Stages the scales of groups g0 .. g0 + wn - 1 (wn = min(left, kWsWin)) of
// the tile's rows, kThreads / kBM threads per row with every copy in flight
// at once (waited for by the caller).
template <int kThreads>
__device__ __forceinline__ void stage_group_scales(float* ws_smem, const float* ws, int G, int d, int row0, int g0,
                                                   int left, int et) {
  const int wn = left < kWsWin ? left : kWsWin;
  constexpr int kTpr = kThreads / kBM;  // threads per row
  const int rl = et / kTpr, rr = row0 + rl;
  float* dst = ws_smem + rl * kWsStride;
  if (rr < d) {
    const float* src = ws + static_cast<size_t>(rr) * G + g0;
    for (int g = et % kTpr; g < wn; g += kTpr) cp_async4(dst + g, src + g);
  } else {
    for (int g = et % kTpr; g < wn; g += kTpr) dst[g] = 0.f;
  }
}

// Every thread of the block, from the producer and the epilogue branches
// alike (named barrier 2).
template <int kThreads>
__device__ __forceinline__ void block_sync() {
  asm volatile("bar.sync 2, %0;" ::"n"(kThreads) : "memory");
}

template <int kEpiWarps>
__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
}

// One CTA's tile and K range: block `blk` of a launch of `a` (split blk %
// splits of tile blk / splits).  The tensor maps live in kernel parameter
// space (grid constants).
template <int kBN>
__device__ __forceinline__ void gemm_tile(const CUtensorMap* map_w, const CUtensorMap* map_x, const Args& a,
                                          int blk) {
  extern __shared__ unsigned char smem_raw[];
  Smem sm = carve(smem_raw, kBN);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // tile / split of this CTA
  const int split = blk % a.splits;
  const int tile = blk / a.splits;
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
  constexpr int kS = stages(kBN);
  constexpr bool kMmaBias = Shape<kBN>::kMmaBias;
  constexpr int kUG = Shape<kBN>::kUnitGroups;    // groups per unit (buffers handed over together)
  constexpr int kUnits = kAccBufs / kUG;          // 4: even, so a unit always has the same owner
  constexpr int kUnitsPerChunk = 2 / kUG;
  constexpr bool kTwoIssuers = kBN <= 32;
  constexpr uint32_t kTmemCols = kAccBufs * kBN;  // 128, 256 or 512: a power of two
  static_assert(kUnits <= kMaxUnits && kUnits % 2 == 0, "units alternate between the two warpgroups");

  if constexpr (kMmaBias) {
    // the offset MMA's operand: every 16-byte chunk the same (generic-proxy
    // writes, made visible to the tensor cores before the block barrier)
    for (uint32_t i = threadIdx.x; i < kBiasTileBytes / 16; i += Shape<kBN>::kThreads)
      reinterpret_cast<uint4*>(sm.bias)[i] = mma_bias_chunk();
    fence_proxy_async_smem();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < kS; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
    }
    for (int i = 0; i < kUnits; ++i) {
      mbar_init(&sm.acc_full[i], 1);
      mbar_init(&sm.acc_empty[i], 4);  // the four warps of the unit's epilogue warpgroup
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

  if (warp < Shape<kBN>::kFirstEpiWarp) {
  if constexpr (Shape<kBN>::kSplitRegs) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsProducer));
  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      // Weights never depend on the previous kernel: fill the ring's weight
      // halves first, then wait for the activations.
      const int first = nchunks < kS ? nchunks : kS;
      for (int c = 0; c < first; ++c) {
        mbar_arrive_expect_tx(&sm.full[c], stage_bytes(kBN));
        tma_load_2d(stage_a(sm, c), map_w, (c_begin + c) * kChunk, row0, &sm.full[c]);
      }
      griddep_wait();
      for (int c = 0; c < first; ++c) tma_load_2d(stage_b(sm, c), map_x, (c_begin + c) * kChunk, tok0, &sm.full[c]);
      for (int c = kS; c < nchunks; ++c) {
        const int st = c % kS;
        if (!mbar_wait_bounded(&sm.empty[st], ((c / kS) - 1) & 1, kWaitLimitNs)) {
          record_device_error(a, kDevMmaTimeout);
          *sm.flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&sm.full[st], stage_bytes(kBN));
        const int kx = (c_begin + c) * kChunk;
        tma_load_2d(stage_a(sm, st), map_w, kx, row0, &sm.full[st]);
        tma_load_2d(stage_b(sm, st), map_x, kx, tok0, &sm.full[st]);
      }
    }
  } else if (warp == 1 || (kTwoIssuers && warp == 2)) {
    // ---------------- MMA issuer(s) ----------------
    // Narrow tiles (kTwoIssuers) have two issuing threads, warp 1 the even
    // chunks and warp 2 the odd ones: one thread's instruction issue bounds
    // them.  The chunks of the two use disjoint units (kUnits is even); a
    // stage passes between them through its full and empty barriers, and a
    // commit tracks only its own thread's MMAs.  Wide tiles are bound by the
    // epilogue, where a second issuer only takes issue slots.  Per chunk: one
    // wait for its stage; per unit one wait for its buffers, per group the
    // offset MMA (128-token tiles) and two K = 32 steps, one commit; one
    // commit for the stage.
    if (lane == 0) {
      const uint32_t idesc = i8_idesc(kBN);
      const uint32_t bias_idesc = u8_idesc(kBN);
      const uint64_t bias_desc = sw32_desc(smem_u32(sm.bias));
      bool ok = true;
      constexpr int kIssuers = kTwoIssuers ? 2 : 1;
      for (int c = warp - 1; c < nchunks && ok; c += kIssuers) {
        const int st = c % kS;
        if (!mbar_wait_bounded(&sm.full[st], (c / kS) & 1, kWaitLimitNs)) {
          ok = false;
          break;
        }
        // descriptor start addresses count 16-byte units: a K step of 32
        // bytes adds 2 (stage bases stay below 2^18 bytes, so no carry)
        const uint64_t a_desc = sw128_desc(smem_u32(stage_a(sm, st)));
        const uint64_t b_desc = sw128_desc(smem_u32(stage_b(sm, st)));
#pragma unroll
        for (int j = 0; j < kUnitsPerChunk; ++j) {
          const int u = c * kUnitsPerChunk + j, ub = u % kUnits;
          // use k of a unit waits for phase k: the epilogue's first arrival
          // (phase 0) or its read of use k - 1
          if (!mbar_wait_bounded(&sm.acc_empty[ub], (u / kUnits) & 1, kWaitLimitNs)) {
            ok = false;
            break;
          }
          tmem_fence_after();
#pragma unroll
          for (int gg = 0; gg < kUG; ++gg) {
            const int g = j * kUG + gg;  // group of the chunk
            const uint32_t d = tmem + static_cast<uint32_t>((ub * kUG + gg) * kBN);
            if constexpr (kMmaBias) mma_i8(d, bias_desc, bias_desc, bias_idesc, false);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              const uint64_t koff = static_cast<uint64_t>(2 * (2 * g + kk));
              mma_i8(d, a_desc + koff, b_desc + koff, idesc, true);
            }
          }
          mma_commit(&sm.acc_full[ub]);
        }
        if (ok) mma_commit(&sm.empty[st]);  // the stage is free once its MMAs have read it
      }
      if (!ok) {
        record_device_error(a, kDevMmaTimeout);
        *sm.flag = 1;
      }
    }
  }
    // the output barriers of the epilogue branch, in the same order
    __syncwarp();
    if (a.cluster > 1) {
      cluster_sync();
      cluster_sync();
    } else {
      block_sync<Shape<kBN>::kThreads>();
    }
  } else {
    if constexpr (Shape<kBN>::kSplitRegs) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsEpilogue));
    // ---------------- epilogue (two warpgroups) ----------------
    const int quad = warp & 3;                                     // TMEM lanes 32*quad .. +31
    const int role = (warp - Shape<kBN>::kFirstEpiWarp) >> 2;      // units u with u % 2 == role
    constexpr int kCols = Shape<kBN>::kCols;
    constexpr int kLd = Shape<kBN>::kLdCols;
    uint64_t acc[kCols / 2];  // fp32 pairs: columns 2j, 2j + 1
#pragma unroll
    for (int j = 0; j < kCols / 2; ++j) acc[j] = 0;
    const uint32_t off_bits = kMmaBias ? kMmaBiasBits : __float_as_uint(kAccBiasF);
    const uint64_t bias2 = f2_pack(off_bits, off_bits);
    const int et = static_cast<int>(threadIdx.x) - Shape<kBN>::kFirstEpiWarp * 32;  // epilogue thread
    const uint32_t tl = tmem + (static_cast<uint32_t>(32 * quad) << 16);
    // Unit u (groups u * kUG ..) fills buffers kUG * (u % kUnits) ..; unit
    // ub always belongs to warpgroup ub % 2 (units alternate and kUnits is
    // even).  Without the offset MMA every buffer starts at the bias.
    if constexpr (!kMmaBias) {
#pragma unroll 1
      for (int b = 0; b < kAccBufs; ++b)
        if ((b / kUG) % 2 == role) tmem_fill_bias<kCols>(tl + static_cast<uint32_t>(b * kBN));
      tmem_wait_st();
      tmem_fence_before();
    }
    __syncwarp();
    if (lane == 0)
      for (int ub = role; ub < kUnits; ub += 2) mbar_arrive(&sm.acc_empty[ub]);
    bool range_ok = true;  // every group scale within the offset MMA's exact range
    auto stage_scales = [&](int g0) {
      stage_group_scales<kEpiWarps * 32>(sm.ws, a.ws, a.G, a.d, row0, 2 * c_begin + g0, ngroups - g0, et);
    };
    // The first window is weight data (no dependency on the previous
    // kernel); xs and the outputs belong to the stream order.
    stage_scales(0);
    griddep_wait();
    if (et < kBN) sm.xs[et] = tok0 + et < a.m ? __ldg(a.xs + tok0 + et) : 0.f;
    cp_async_wait_all();
    epi_sync<kEpiWarps>();
    bool ok = true;
    for (int w0 = 0; w0 < ngroups; w0 += kWsWin) {  // windows of group scales (whole unit pairs)
      if (w0 > 0) {
        epi_sync<kEpiWarps>();  // both warpgroups are done with the previous window
        stage_scales(w0);
        cp_async_wait_all();
        epi_sync<kEpiWarps>();
      }
      const int wend = ngroups - w0 < kWsWin ? ngroups : w0 + kWsWin;
      // this warpgroup's units of the window (unit u: groups u * kUG ..
      // in buffers kUG * (u % kUnits) ..); after a timeout the warp keeps
      // walking the windows without waiting, so that both warpgroups meet
      // the same barriers
      for (int u = w0 / kUG + role; u * kUG < wend; u += 2) {
        const int ub = u % kUnits;
        const float* wrow = sm.ws + (32 * quad + lane) * kWsStride + (u * kUG - w0);
        if (ok && !mbar_wait_bounded(&sm.acc_full[ub], (u / kUnits) & 1, kWaitLimitNs)) ok = false;
        if (!ok) continue;
        tmem_fence_after();
        // The unit's groups as one software pipeline of kLd-column loads:
        // load q + 1 is issued as soon as load q has landed, so its latency
        // overlaps q's arithmetic (one exposed load per unit).
        {
          static_assert(kLd == 16, "pipelined loads of 16 columns");
          constexpr int kL = kCols / kLd;  // loads per group
          const uint32_t base = tl + static_cast<uint32_t>(ub * kUG * kBN);
          uint64_t w2[kUG];
#pragma unroll
          for (int gg = 0; gg < kUG; ++gg) {
            float w = wrow[gg];
            if constexpr (kMmaBias) {
              const float ws = w * __uint_as_float(kMmaScaleIn);  // exact below 2^38
              range_ok &= !(isinf(ws) && isfinite(w));
              w = ws;
            }
            w2[gg] = f2_pack(__float_as_uint(w), __float_as_uint(w));
          }
          uint32_t ra[kLd], rb[kLd];
          tmem_ld16(base, ra);
#pragma unroll
          for (int q = 0; q < kUG * kL; ++q) {
            uint32_t(&cur)[kLd] = (q & 1) ? rb : ra;
            uint32_t(&nxt)[kLd] = (q & 1) ? ra : rb;
            tmem_wait_ld16(cur);
            if (q + 1 < kUG * kL) {
              const int q1 = q + 1;
              tmem_ld16(base + static_cast<uint32_t>((q1 / kL) * kBN + kLd * (q1 % kL)), nxt);
            }
            const int col = (q % kL) * (kLd / 2);
#pragma unroll
            for (int j = 0; j < kLd / 2; ++j)
              acc[col + j] = f2_unbias_fma(f2_pack(cur[2 * j], cur[2 * j + 1]), bias2, w2[q / kL], acc[col + j]);
          }
          if constexpr (!kMmaBias) {
            // the unit's buffers ready for their next use
#pragma unroll
            for (int gg = 0; gg < kUG; ++gg) tmem_fill_bias<kCols>(base + static_cast<uint32_t>(gg * kBN));
            tmem_wait_st();
          }
        }
        // the buffers go back to the MMA warp once read (and refilled)
        tmem_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.acc_empty[ub]);
      }
    }
    if (!ok) {
      record_device_error(a, kDevMmaTimeout);
      *sm.flag = 1;
    }
    if constexpr (kMmaBias) {
      if (!range_ok) {
        record_device_error(a, kDevScaleRange);
        *sm.flag = 1;
      }
    }
    epi_sync<kEpiWarps>();
    // Every load has landed and every MMA that read the ring has
    // completed, so the ring takes the finished tile as [token][row]: the
    // two warpgroups' sums added in a fixed order (warpgroup 1, then 2),
    // scaled by xs[t] when the tile is the whole sum, the raw partial sum of
    // this block's K range otherwise.
    const bool good = *sm.flag == 0;
    float* tile = reinterpret_cast<float*>(sm.ring);
    const int r_local = 32 * quad + lane;
    // sums of the offset-MMA path are kept scaled by 2^-59 (exact)
    const float out_scale = kMmaBias ? __uint_as_float(kMmaScaleOut) : 1.f;
    if (good && role == 0) {
#pragma unroll
      for (int j = 0; j < kCols / 2; ++j) {
        float v0, v1;
        f2_unpack(acc[j], v0, v1);
        v0 *= out_scale;
        v1 *= out_scale;
        tile[(2 * j) * kBM + r_local] = v0;
        tile[(2 * j + 1) * kBM + r_local] = v1;
      }
    }
    epi_sync<kEpiWarps>();
    if (good && role == 1) {
      const bool whole = a.splits == 1;
#pragma unroll
      for (int j = 0; j < kCols / 2; ++j) {
        float v0, v1;
        f2_unpack(acc[j], v0, v1);
        v0 *= out_scale;
        v1 *= out_scale;
        float* t0 = tile + (2 * j) * kBM + r_local;
        float* t1 = tile + (2 * j + 1) * kBM + r_local;
        const float s0 = *t0 + v0, s1 = *t1 + v1;
        *t0 = whole ? s0 * sm.xs[2 * j] : s0;
        *t1 = whole ? s1 * sm.xs[2 * j + 1] : s1;
      }
    }

    // ---------------- output (every thread of the block takes part in the barriers) ----------------
    __syncwarp();
    if (a.cluster > 1) cluster_sync(); else block_sync<Shape<kBN>::kThreads>();
    constexpr int kEpiThreads = Shape<kBN>::kEpiWarps * 32;
    constexpr int kQuads = kBN * kBM / 4;  // float4s in the tile; 32 per token
    const uint32_t tile_s = smem_u32(sm.ring);
    if (a.cluster > 1) {
      // Block `split` of the cluster sums its share of the tile over the
      // cluster's partial tiles in split order (deterministic), scales by
      // xs[t] and writes Y.
      const int s = a.cluster;
      bool all_good = true;
      for (int p = 0; p < s; ++p) all_good &= ld_cluster_s32(cluster_peer(smem_u32(sm.flag), p)) == 0;
      if (all_good) {
        // This thread's float4s of the share, q = q0 + et + k * kEpiThreads:
        // per partial tile, every load is issued before the first is used (one
        // remote round trip per split instead of one per float4), summed in
        // split order.
        constexpr int kMaxIt = (kQuads + kEpiThreads - 1) / kEpiThreads;
        const int q0 = split * kQuads / s, q1 = (split + 1) * kQuads / s;
        float4 v[kMaxIt];
#pragma unroll
        for (int k = 0; k < kMaxIt; ++k) v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int p = 0; p < s; ++p) {
          const uint32_t peer_tile = cluster_peer(tile_s, p);
          float4 u[kMaxIt];
#pragma unroll
          for (int k = 0; k < kMaxIt; ++k) {
            const int q = q0 + et + k * kEpiThreads;
            u[k] = q < q1 ? ld_cluster_f4(peer_tile + 16u * q) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int k = 0; k < kMaxIt; ++k) {
            v[k].x += u[k].x;
            v[k].y += u[k].y;
            v[k].z += u[k].z;
            v[k].w += u[k].w;
          }
        }
#pragma unroll
        for (int k = 0; k < kMaxIt; ++k) {
          const int q = q0 + et + k * kEpiThreads;
          const int j = q >> 5, t = tok0 + j;
          if (q >= q1 || t >= a.m) continue;
          const float x = sm.xs[j];
          store_out4(a.y, a, t, row0 + 4 * (q & 31),
                     make_float4(v[k].x * x, v[k].y * x, v[k].z * x, v[k].w * x));
        }
      }
    } else if (*sm.flag == 0) {
      // the whole sum (splits == 1), or this split's partial, which
      // splitk_reduce_kernel sums in split order
      float* dst = a.splits == 1 ? a.y : a.partial + static_cast<size_t>(split) * a.m * a.d;
      const float4* tile4 = reinterpret_cast<const float4*>(sm.ring);
      for (int q = et; q < kQuads; q += kEpiThreads) {
        const int j = q >> 5, t = tok0 + j;
        if (t < a.m) store_out4(dst, a, t, row0 + 4 * (q & 31), tile4[q]);
      }
    }
    // no block leaves while the others may still read its tile
    if (a.cluster > 1) cluster_sync();
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

template <int kBN>
__global__ void __launch_bounds__(Shape<kBN>::kThreads, 1)
    gemm_w8a8_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                        const __grid_constant__ Args a) {
  gemm_tile<kBN>(&map_w, &map_x, a, static_cast<int>(blockIdx.x));
}

// Several independent GEMMs with the same token count in one launch: op o
// owns blocks [base[o], base[o + 1]) (a multiple of its split count, so a
// cluster never spans two ops).
constexpr int kMaxGroupOps = 8;
struct GroupArgs {
  CUtensorMap mw[kMaxGroupOps];
  CUtensorMap mx[kMaxGroupOps];
  Args op[kMaxGroupOps];
  int base[kMaxGroupOps + 1];
  int count;
};

template <int kBN>
__global__ void __launch_bounds__(Shape<kBN>::kThreads, 1)
    gemm_w8a8_tc_group_kernel(const __grid_constant__ GroupArgs g) {
  int o = 0;
  while (o + 1 < g.count && static_cast<int>(blockIdx.x) >= g.base[o + 1]) ++o;
  gemm_tile<kBN>(&g.mw[o], &g.mx[o], g.op[o], static_cast<int>(blockIdx.x) - g.base[o]);
}

// ---------------------------------------------------------------------------
// Persistent whole tiles (128 tokens per tile).  One CTA per SM walks a list
// of output tiles made on the host (whole K per tile, no split; largest
// first onto the least-loaded CTA), and its TMA, MMA and epilogue counters
// run on across tile boundaries: the next tile's loads and MMAs proceed
// while the epilogue finishes the current one, and the block's set-up
// (barriers, tensor memory, the offset tile) happens once per launch.
//   * warp 0 streams 32 KB stages (128 weight rows x 128 B and 128 tokens x
//     128 B) into a ring of kPStages;
//   * warps 1 and 2 issue the MMAs of alternate chunks (one thread's
//     instruction issue would bound the loop): per 64-column group the
//     offset MMA and two K = 32 steps into one of kPBufs single-group
//     buffers of 128 columns (a chunk's two groups fill buffers 0-1 or 2-3,
//     so the two issuers never share one);
//   * the epilogue warpgroups split the tile by token columns (warpgroup w
//     the 64 tokens 64 w ..), so every epilogue thread ends a tile holding
//     the complete sums of its weight row for its 64 tokens, and stores them
//     straight to Y (a warp writes 32 consecutive rows of one token: 128
//     contiguous bytes).  Group scales come from global memory, a few chunks
//     ahead of their use.
// ---------------------------------------------------------------------------
constexpr int kPStages = 6;
constexpr uint32_t kPStage = kStageA + 128u * kChunk;   // 32 KB
constexpr int kPBufs = 4;                               // 4 x 128 = 512 tensor-memory columns
constexpr int kPCols = 64;                              // token columns per epilogue warpgroup
constexpr int kPWsAhead = 4;                            // chunks of group scales in flight
constexpr int kPMaxUnits = 4096;                        // tiles in one launch
constexpr int kPMaxCtas = 256;                          // at least the SM count
constexpr int kPThreads = 384;
constexpr int kPStreams = 1;  // tile lists per CTA
constexpr uint32_t kPSmemBytes = 1024u + kPStages * kPStage + kBiasTileBytes + 256u;

struct POp {
  float* y;
  const float* xs;
  const float* ws;
  int m, n, d, G, tiles_n, chunks;
};
struct PArgs {
  CUtensorMap mw[kMaxGroupOps];
  CUtensorMap mx[kMaxGroupOps];
  POp op[kMaxGroupOps];
  unsigned int* err;
  unsigned short first[kPStreams * kPMaxCtas + 1];  // CTA c runs unit[first[c] .. first[c + 1])
  unsigned short unit[kPMaxUnits];      // (op << 12) | tile, tile = tile_m * tiles_n + tile_n
};

static_assert(kPSmemBytes <= 232448, "shared memory per block");
static_assert(sizeof(PArgs) <= 32764, "kernel parameter space");
static_assert(kPStages % 2 == 0 && kPBufs % 4 == 0, "alternate chunks keep to their own stages and buffers");

struct PTile {
  int o, row0, tok0, chunks;
};
__device__ __forceinline__ PTile p_tile(const PArgs& p, int i) {
  const unsigned u = p.unit[i];
  PTile t;
  t.o = static_cast<int>(u >> 12);
  const int tile = static_cast<int>(u & 0xFFFu);
  const int tn = p.op[t.o].tiles_n;
  t.row0 = (tile / tn) * kBM;
  t.tok0 = (tile % tn) * 128;
  t.chunks = p.op[t.o].chunks;
  return t;
}

__device__ __forceinline__ void p_record_error(const PArgs& p, unsigned int code) {
  if (p.err) atomicCAS(p.err, 0u, code);
}

// The group scales of chunk c (groups 2c, 2c + 1) of one weight row.
__device__ __forceinline__ float2 p_ws(const float2* row, bool in, int c, int chunks) {
  return in && c < chunks ? __ldg(row + c) : make_float2(0.f, 0.f);
}

__global__ void __launch_bounds__(kPThreads, 1) gemm_w8a8_persistent_kernel(const __grid_constant__ PArgs p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* ring = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~static_cast<uintptr_t>(1023u));
  unsigned char* bias = ring + kPStages * kPStage;
  uint64_t* full = reinterpret_cast<uint64_t*>(bias + kBiasTileBytes);
  uint64_t* empty = full + kPStages;
  uint64_t* acc_full = empty + kPStages;
  uint64_t* acc_empty = acc_full + kPBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + kPBufs);
  volatile int* broken = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u_begin = p.first[blockIdx.x], u_end = p.first[blockIdx.x + 1];

  for (uint32_t i = threadIdx.x; i < kBiasTileBytes / 16; i += kPThreads)
    reinterpret_cast<uint4*>(bias)[i] = mma_bias_chunk();
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    for (int i = 0; i < kPStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < kPBufs; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);  // every epilogue warp reads every buffer
    }
    *broken = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kPBufs * 128u)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_launch_dependents();

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsProducer));
    if (warp == 0 && lane == 0) {
      // ---------------- TMA producer ----------------
      bool ok = true;
      // The first tile's weight chunks that fit the ring go out before the
      // wait for the previous kernel (weights never depend on it).
      int pre = 0;
      if (u_begin < u_end) {
        const PTile f = p_tile(p, u_begin);
        pre = f.chunks < kPStages ? f.chunks : kPStages;
        for (int c = 0; c < pre; ++c) {
          mbar_arrive_expect_tx(&full[c], kPStage);
          tma_load_2d(ring + c * kPStage, &p.mw[f.o], c * kChunk, f.row0, &full[c]);
        }
      }
      griddep_wait();
      int gc = 0;  // chunk counter over the whole tile list
      for (int i = u_begin; i < u_end && ok; ++i) {
        const PTile t = p_tile(p, i);
        for (int c = 0; c < t.chunks; ++c, ++gc) {
          const int st = gc % kPStages;
          unsigned char* sa = ring + st * kPStage;
          if (gc < pre) {
            tma_load_2d(sa + kStageA, &p.mx[t.o], c * kChunk, t.tok0, &full[st]);
            continue;
          }
          if (gc >= kPStages && !mbar_wait_bounded(&empty[st], ((gc / kPStages) - 1) & 1, kWaitLimitNs)) {
            ok = false;
            break;
          }
          if (*broken) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[st], kPStage);
          tma_load_2d(sa, &p.mw[t.o], c * kChunk, t.row0, &full[st]);
          tma_load_2d(sa + kStageA, &p.mx[t.o], c * kChunk, t.tok0, &full[st]);
        }
      }
      if (!ok) {
        p_record_error(p, kDevMmaTimeout);
        *broken = 1;
      }
    } else if ((warp == 1 || warp == 2) && lane == 0) {
      // ---------------- MMA issuers: warp 1 the even chunks, warp 2 the odd ----------------
      const uint32_t idesc = i8_idesc(128);
      const uint32_t bias_idesc = u8_idesc(128);
      const uint64_t bias_desc = sw32_desc(smem_u32(bias));
      bool ok = true;
      int gc = 0, gu = 0;  // chunk and group counters over the whole tile list
      for (int i = u_begin; i < u_end && ok; ++i) {
        const PTile t = p_tile(p, i);
        for (int c = 0; c < t.chunks && ok; ++c, ++gc) {
          if ((gc & 1) != warp - 1) {
            gu += 2;
            continue;
          }
          const int st = gc % kPStages;
          if (!mbar_wait_bounded(&full[st], (gc / kPStages) & 1, kWaitLimitNs) || *broken) {
            ok = false;
            break;
          }
          const uint64_t a_desc = sw128_desc(smem_u32(ring + st * kPStage));
          const uint64_t b_desc = sw128_desc(smem_u32(ring + st * kPStage + kStageA));
#pragma unroll
          for (int g = 0; g < 2; ++g, ++gu) {
            const int ub = gu % kPBufs;
            if (!mbar_wait_bounded(&acc_empty[ub], (gu / kPBufs) & 1, kWaitLimitNs)) {
              ok = false;
              break;
            }
            tmem_fence_after();
            const uint32_t d = tmem + static_cast<uint32_t>(ub * 128);
            mma_i8(d, bias_desc, bias_desc, bias_idesc, false);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              const uint64_t koff = static_cast<uint64_t>(2 * (2 * g + kk));
              mma_i8(d, a_desc + koff, b_desc + koff, idesc, true);
            }
            mma_commit(&acc_full[ub]);
          }
          if (ok) mma_commit(&empty[st]);
        }
      }
      if (!ok) {
        p_record_error(p, kDevMmaTimeout);
        *broken = 1;
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsEpilogue));
    // ---------------- epilogue: 8 warps, token columns by warpgroup ----------------
    const int quad = warp & 3;
    const int role = (warp - 4) >> 2;
    const int r_local = 32 * quad + lane;
    const uint32_t tl = tmem + (static_cast<uint32_t>(32 * quad) << 16) + static_cast<uint32_t>(role * kPCols);
    const uint64_t off2 = f2_pack(kMmaBiasBits, kMmaBiasBits);
    const float scale_in = __uint_as_float(kMmaScaleIn);
    const float scale_out = __uint_as_float(kMmaScaleOut);
    __syncwarp();
    if (lane == 0)
      for (int ub = 0; ub < kPBufs; ++ub) mbar_arrive(&acc_empty[ub]);  // every buffer starts free
    griddep_wait();  // xs and the outputs belong to the stream order
    bool ok = true, range_ok = true;
    int gu = 0;
    for (int i = u_begin; i < u_end; ++i) {
      const PTile t = p_tile(p, i);
      const POp& op = p.op[t.o];
      const int row = t.row0 + r_local;
      const bool row_in = row < op.d;  // rows past d read zeros (TMA fill) and are not stored
      const float2* wsrow = reinterpret_cast<const float2*>(op.ws + static_cast<size_t>(row_in ? row : 0) * op.G);
      static_assert(kPWsAhead == 4, "four chunks of scales in flight");
      float2 w0 = p_ws(wsrow, row_in, 0, t.chunks), w1 = p_ws(wsrow, row_in, 1, t.chunks);
      float2 w2 = p_ws(wsrow, row_in, 2, t.chunks), w3 = p_ws(wsrow, row_in, 3, t.chunks);
      uint64_t acc[kPCols / 2];
#pragma unroll
      for (int j = 0; j < kPCols / 2; ++j) acc[j] = 0;
#pragma unroll 1
      for (int c = 0; c < t.chunks; ++c) {
        const float2 wc = w0;
        w0 = w1;
        w1 = w2;
        w2 = w3;
        w3 = p_ws(wsrow, row_in, c + kPWsAhead, t.chunks);
#pragma unroll
        for (int g = 0; g < 2; ++g, ++gu) {
          const int ub = gu % kPBufs;
          if (ok && (!mbar_wait_bounded(&acc_full[ub], (gu / kPBufs) & 1, kWaitLimitNs) || *broken)) ok = false;
          if (!ok) continue;
          tmem_fence_after();
          uint32_t ra[32], rb[32];
          tmem_ld32(tl + static_cast<uint32_t>(ub * 128), ra);
          tmem_ld32(tl + static_cast<uint32_t>(ub * 128 + 32), rb);
          tmem_wait_ld16(*reinterpret_cast<uint32_t(*)[16]>(ra));
          tmem_wait_ld16(*reinterpret_cast<uint32_t(*)[16]>(ra + 16));
          tmem_wait_ld16(*reinterpret_cast<uint32_t(*)[16]>(rb));
          tmem_wait_ld16(*reinterpret_cast<uint32_t(*)[16]>(rb + 16));
          // the buffer is back with the MMA warp as soon as it is in registers
          tmem_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[ub]);
          const float w = g ? wc.y : wc.x;
          const float wsc = w * scale_in;  // exact below 2^38
          range_ok &= !(isinf(wsc) && isfinite(w));
          const uint64_t w2p = f2_pack(__float_as_uint(wsc), __float_as_uint(wsc));
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[j] = f2_unbias_fma(f2_pack(ra[2 * j], ra[2 * j + 1]), off2, w2p, acc[j]);
#pragma unroll
          for (int j = 0; j < 16; ++j)
            acc[16 + j] = f2_unbias_fma(f2_pack(rb[2 * j], rb[2 * j + 1]), off2, w2p, acc[16 + j]);
        }
      }
      if (ok && range_ok && row_in) {
        // Y[t][row] for this warpgroup's 64 tokens: (sum * 2^59) * xs[t]
        const int tb = t.tok0 + role * kPCols;
#pragma unroll
        for (int j = 0; j < kPCols / 2; ++j) {
          float v0, v1;
          f2_unpack(acc[j], v0, v1);
          const int t0 = tb + 2 * j;
          if (t0 < op.m) op.y[static_cast<size_t>(t0) * op.d + row] = (v0 * scale_out) * __ldg(op.xs + t0);
          if (t0 + 1 < op.m) op.y[static_cast<size_t>(t0 + 1) * op.d + row] = (v1 * scale_out) * __ldg(op.xs + t0 + 1);
        }
      }
    }
    if (!ok) {
      p_record_error(p, kDevMmaTimeout);
      *broken = 1;
    }
    if (!range_ok) p_record_error(p, kDevScaleRange);
  }

  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPBufs * 128u) : "memory");
}

// Split-K: y[t][r] = xs[t] * sum_s partial[s][t][r], the splits summed in split
// order (deterministic), over the whole GPU at once.  Launched right after
// the GEMM (programmatic dependent launch): the partials are read only after
// griddepcontrol.wait.
constexpr int kReduceThreads = 256;
constexpr int kReduceElems = 4;   // consecutive outputs per thread (one float4)
constexpr int kReduceBatch = 8;   // splits whose loads are in flight at once

__global__ void __launch_bounds__(kReduceThreads)
    splitk_reduce_kernel(float* y, const float* partial, const float* xs, int splits, int m, int d, int vec4) {
  griddep_wait();
  const size_t md = static_cast<size_t>(m) * d;
  const size_t i0 = (static_cast<size_t>(blockIdx.x) * kReduceThreads + threadIdx.x) * kReduceElems;
  if (i0 >= md) return;
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (vec4 && i0 + kReduceElems <= md) {
    // d % 4 == 0: the four outputs share a token
    for (int s0 = 0; s0 < splits; s0 += kReduceBatch) {
      float4 p[kReduceBatch];
#pragma unroll
      for (int b = 0; b < kReduceBatch; ++b)
        if (s0 + b < splits) p[b] = __ldcg(reinterpret_cast<const float4*>(partial + static_cast<size_t>(s0 + b) * md + i0));
#pragma unroll
      for (int b = 0; b < kReduceBatch; ++b)
        if (s0 + b < splits) {
          v.x += p[b].x;
          v.y += p[b].y;
          v.z += p[b].z;
          v.w += p[b].w;
        }
    }
    const float x = __ldg(xs + i0 / d);
    *reinterpret_cast<float4*>(y + i0) = make_float4(v.x * x, v.y * x, v.z * x, v.w * x);
    return;
  }
  float e[kReduceElems] = {0.f, 0.f, 0.f, 0.f};
  for (int sp = 0; sp < splits; ++sp)
#pragma unroll
    for (int k = 0; k < kReduceElems; ++k)
      if (i0 + k < md) e[k] += __ldcg(partial + static_cast<size_t>(sp) * md + i0 + k);
#pragma unroll
  for (int k = 0; k < kReduceElems; ++k) {
    const size_t i = i0 + k;
    if (i < md) y[i] = e[k] * __ldg(xs + i / d);
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
  int cluster;  // > 1: the splits of a tile form one cluster (no workspace)
};

// K splits that fill the SMs in one wave, keeping at least two 128-byte chunks
// (four groups) per split.
Plan plan(int m, int n, int d, int sm_count) {
  Plan p;
  p.bn = m <= 16 ? 16 : (m <= 32 ? 32 : (m <= 64 ? 64 : 128));
  p.tiles_m = (d + kBM - 1) / kBM;
  p.tiles_n = (m + p.bn - 1) / p.bn;
  p.chunks = n / kChunk;
  const int tiles = p.tiles_m * p.tiles_n;
  int splits = sm_count / tiles;
  if (splits > p.chunks / 2) splits = p.chunks / 2;
  if (splits < 1) splits = 1;
  p.splits = splits;
  p.cluster = 1;
  return p;
}

template <int kBN>
cudaError_t prepare_bn() {
  return ensure_dynamic_smem(reinterpret_cast<const void*>(gemm_w8a8_tc_kernel<kBN>), smem_bytes(kBN));
}

// How many clusters of `size` blocks of the kBN kernel the current device
// runs at once (cached per device, tile width and size).
constexpr int kMaxCluster = 16;
constexpr int kMaxDevicesTc = 64;

template <int kBN>
int max_active_clusters(int device, int size) {
  static std::mutex mu;
  static int cache[kMaxDevicesTc][kMaxCluster + 1];
  static bool init = false;
  std::lock_guard<std::mutex> lock(mu);
  if (!init) {
    for (auto& row : cache)
      for (int& v : row) v = -1;
    init = true;
  }
  if (device < 0 || device >= kMaxDevicesTc || size < 1 || size > kMaxCluster) return 0;
  int& c = cache[device][size];
  if (c >= 0) return c;
  c = 0;
  const void* fn = reinterpret_cast<const void*>(gemm_w8a8_tc_kernel<kBN>);
  if (prepare_bn<kBN>() != cudaSuccess) return 0;
  if (size > 8 && cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(size);
  cfg.blockDim = dim3(Shape<kBN>::kThreads);
  cfg.dynamicSmemBytes = smem_bytes(kBN);
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = size;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_w8a8_tc_kernel<kBN>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  c = n;
  return c;
}

int max_active_clusters_bn(int bn, int device, int size) {
  switch (bn) {
    case 16: return max_active_clusters<16>(device, size);
    case 32: return max_active_clusters<32>(device, size);
    case 64: return max_active_clusters<64>(device, size);
    default: return max_active_clusters<128>(device, size);
  }
}

// How the K splits of a tile are summed: inside a cluster over shared memory
// (no second kernel) with the largest cluster size whose clusters all fit on
// the GPU at once, or through the workspace with the split count that fills
// the SMs and a second kernel.  The estimate behind the choice: a block's
// time grows with its K chunks (about 0.9 us per 128-byte chunk at 128
// tokens per tile, 0.5 us at 16-32 tokens on a B200), and the second kernel
// with the launch gaps around it costs about 4.5 us.
Plan choose(int m, int n, int d, const DeviceInfo& dev, bool have_ws) {
  Plan p = plan(m, n, d, dev.sm_count);
  const int want = p.splits;
  const int tiles = p.tiles_m * p.tiles_n;
  int s = (launch_flags() & MLI_LAUNCH_NO_CLUSTER) ? 1 : (want < kMaxCluster ? want : kMaxCluster);
  while (s > 1 && max_active_clusters_bn(p.bn, dev.device, s) < tiles) --s;
  bool cluster = s == want || !have_ws;
  if (!cluster && s > 1) {
    const double per_chunk_us = p.bn >= 128 ? 0.9 : (p.bn >= 64 ? 0.6 : 0.5);
    const double t_cluster = ((p.chunks + s - 1) / s) * per_chunk_us;
    const double t_ws = ((p.chunks + want - 1) / want) * per_chunk_us + 4.5;
    cluster = t_cluster <= t_ws;
  }
  if (cluster) {
    p.splits = s;
    p.cluster = s;
  }
  return p;
}

// The setmaxnreg split must fit the registers the block is launched with:
// an increase beyond them would wait forever.  Checked once per kernel
// against the compiled register count.
template <int kBN, typename K>
bool register_split_fits(K kernel) {
  static const bool fits = [kernel]() {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kernel) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    return !Shape<kBN>::kSplitRegs || fa.numRegs * Shape<kBN>::kThreads >= kRegsBlock;
  }();
  return fits;
}

template <int kBN>
cudaError_t launch_bn(const CUtensorMap& mw, const CUtensorMap& mx, const Args& a, int grid,
                      cudaStream_t stream) {
  if (!register_split_fits<kBN>(gemm_w8a8_tc_kernel<kBN>)) return cudaErrorInvalidConfiguration;
  cudaError_t e = prepare_bn<kBN>();
  if (e != cudaSuccess) return e;
  if (a.cluster > 8) {
    e = cudaFuncSetAttribute(reinterpret_cast<const void*>(gemm_w8a8_tc_kernel<kBN>),
                             cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
  return launch_clustered(gemm_w8a8_tc_kernel<kBN>, dim3(grid), dim3(Shape<kBN>::kThreads), smem_bytes(kBN),
                          stream, true, static_cast<unsigned>(a.cluster), mw, mx, a);
}

template <int kBN>
cudaError_t launch_group_bn(const GroupArgs& g, int grid, int cluster, cudaStream_t stream) {
  if (!register_split_fits<kBN>(gemm_w8a8_tc_group_kernel<kBN>)) return cudaErrorInvalidConfiguration;
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(gemm_w8a8_tc_group_kernel<kBN>), smem_bytes(kBN));
  if (e != cudaSuccess) return e;
  return launch_clustered(gemm_w8a8_tc_group_kernel<kBN>, dim3(grid), dim3(Shape<kBN>::kThreads), smem_bytes(kBN),
                          stream, true, static_cast<unsigned>(cluster), g);
}

// ---------------------------------------------------------------------------
// Persistent plan: whole tiles, each costing its K chunks plus one chunk of
// set-up and output, largest first onto the least-loaded CTA (ties to the
// lowest CTA).  Taken when every SM gets a tile and the busiest CTA carries
// at most kPMaxImbalance times the ideal share of all the SMs; otherwise the
// split-K kernels fill the GPU better.
// ---------------------------------------------------------------------------
constexpr double kPMaxImbalance = 1.3;
constexpr int kPTileOverhead = 1;

struct PChoice {
  bool use = false;
  int ctas = 0, units = 0;
  long long makespan = 0, total = 0;
};

PChoice persistent_plan(const mli_gemm_op* ops, int count, int m, const DeviceInfo& dev, PArgs* pa) {
  PChoice r;
  if (m <= 64 || count < 1 || count > kMaxGroupOps || (launch_flags() & MLI_LAUNCH_NO_PERSISTENT)) return r;
  const int tiles_n = (m + 127) / 128;
  int order[kMaxGroupOps];
  for (int i = 0; i < count; ++i) {
    if (ops[i].n % kChunk != 0 || !aligned(ops[i].w_s, 8)) return r;
    const long long tiles = static_cast<long long>((ops[i].d + kBM - 1) / kBM) * tiles_n;
    if (tiles > 4096 || r.units + tiles > kPMaxUnits) return r;
    r.units += static_cast<int>(tiles);
    r.total += tiles * (ops[i].n / kChunk + kPTileOverhead);
    order[i] = i;
  }
  for (int i = 1; i < count; ++i)  // ops by tile cost, largest first (stable)
    for (int j = i; j > 0 && ops[order[j]].n > ops[order[j - 1]].n; --j) {
      const int t = order[j];
      order[j] = order[j - 1];
      order[j - 1] = t;
    }
  r.ctas = r.units < dev.sm_count ? r.units : dev.sm_count;
  if (r.ctas > kPMaxCtas) r.ctas = kPMaxCtas;
  if (r.ctas < 1) return r;
  // min-heap of (load, cta)
  static thread_local long long load[kPMaxCtas];
  static thread_local long long sload[kPStreams * kPMaxCtas];
  static thread_local int heap[kPMaxCtas];
  static thread_local unsigned short assign[kPMaxUnits];
  static thread_local unsigned short code[kPMaxUnits];
  const int H = r.ctas;
  auto less = [&](int a, int b) { return load[a] < load[b] || (load[a] == load[b] && a < b); };
  for (int c = 0; c < H; ++c) {
    load[c] = 0;
    for (int k = 0; k < kPStreams; ++k) sload[kPStreams * c + k] = 0;
    heap[c] = c;  // all loads zero: index order is a valid heap
  }
  int u = 0;
  for (int k = 0; k < count; ++k) {
    const int o = order[k];
    const long long cost = ops[o].n / kChunk + kPTileOverhead;
    const int tiles = ((ops[o].d + kBM - 1) / kBM) * tiles_n;
    for (int tile = 0; tile < tiles; ++tile, ++u) {
      const int c = heap[0];
      const int v = kPStreams == 1 ? c : kPStreams * c + (sload[kPStreams * c + 1] < sload[kPStreams * c] ? 1 : 0);
      assign[u] = static_cast<unsigned short>(v);
      code[u] = static_cast<unsigned short>((k << 12) | tile);  // op slot k of the launch
      sload[v] += cost;
      load[c] += cost;
      // sift down
      int i = 0;
      for (;;) {
        const int l = 2 * i + 1, rr = l + 1;
        int m = i;
        if (l < H && less(heap[l], heap[m])) m = l;
        if (rr < H && less(heap[rr], heap[m])) m = rr;
        if (m == i) break;
        const int t = heap[i];
        heap[i] = heap[m];
        heap[m] = t;
        i = m;
      }
    }
  }
  for (int c = 0; c < H; ++c) r.makespan = load[c] > r.makespan ? load[c] : r.makespan;
  r.use = r.units >= dev.sm_count &&
          static_cast<double>(r.makespan) <= kPMaxImbalance * static_cast<double>(r.total) / dev.sm_count;
  if (!r.use || !pa) return r;
  // units grouped by CTA, each CTA's in the order assigned
  const int V = kPStreams * H;
  int cnt[kPStreams * kPMaxCtas + 1] = {};
  for (int i = 0; i < r.units; ++i) ++cnt[assign[i] + 1];
  for (int v = 0; v < V; ++v) cnt[v + 1] += cnt[v];
  for (int v = 0; v <= V; ++v) pa->first[v] = static_cast<unsigned short>(cnt[v]);
  for (int i = 0; i < r.units; ++i) pa->unit[cnt[assign[i]]++] = code[i];
  // op slots in the launch follow the cost order
  for (int k = 0; k < count; ++k) {
    const mli_gemm_op& op = ops[order[k]];
    if (!make_map(&pa->mw[k], op.w_q, op.d, op.n, kBM) || !make_map(&pa->mx[k], op.xq, m, op.n, 128)) {
      r.use = false;
      return r;
    }
    POp& po = pa->op[k];
    po.y = op.y;
    po.xs = op.xs;
    po.ws = op.w_s;
    po.m = m;
    po.n = op.n;
    po.d = op.d;
    po.G = op.n / 64;
    po.tiles_n = tiles_n;
    po.chunks = op.n / kChunk;
  }
  pa->err = device_error_word();
  return r;
}

// Plans and launches the persistent kernel: returns -1 (nothing launched)
// when the split-K kernels are the better plan, else the status.
int launch_persistent(const mli_gemm_op* ops, int count, int m, const DeviceInfo& dev, cudaStream_t stream) {
  static thread_local PArgs pa;
  const PChoice ch = persistent_plan(ops, count, m, dev, &pa);
  if (!ch.use) return -1;
  static const bool fits = []() {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, gemm_w8a8_persistent_kernel) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    return fa.numRegs * kPThreads >= kRegsBlock;
  }();
  if (!fits) return check_cuda(cudaErrorInvalidConfiguration);
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(gemm_w8a8_persistent_kernel), kPSmemBytes);
  if (e != cudaSuccess) return check_cuda(e);
  return check_cuda(launch(gemm_w8a8_persistent_kernel, dim3(ch.ctas), dim3(kPThreads), kPSmemBytes, stream, true, pa));
}

// ---------------------------------------------------------------------------
// The int8 tensor-core roof of this GPU (mli_debug_int8_mma_peak): every CTA
// issues back-to-back kind::i8 MMAs (M = 128, N = kN, K = 32) from one thread
// on operands resident in shared memory (zeros: the values do not change the
// rate), alternating between two accumulators, with no loads and no
// epilogue -- the denominator the batched path's tensor utilisation is
// measured against.
// ---------------------------------------------------------------------------
template <int kN>
__global__ void __launch_bounds__(128, 1) mma_peak_kernel(int iters, unsigned int* err) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~static_cast<uintptr_t>(1023u));
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;
  constexpr uint32_t kBytes = kStageA + kN * kChunk;
  for (uint32_t i = threadIdx.x * 16u; i < kBytes; i += 128u * 16u)
    *reinterpret_cast<uint4*>(base + i) = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();  // the zeros are visible to the tensor cores
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  constexpr uint32_t kCols = 2 * kN;
  if ((threadIdx.x >> 5) == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = tmem_base;
  if (threadIdx.x == 0) {
    const uint32_t idesc = i8_idesc(kN);
    const uint64_t a_desc = sw128_desc(smem_u32(base));
    const uint64_t b_desc = sw128_desc(smem_u32(base + kStageA));
    for (int it = 0; it < iters; ++it) {
      const uint32_t d = tmem + static_cast<uint32_t>((it & 1) * kN);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) mma_i8(d, a_desc + 2 * kk, b_desc + 2 * kk, idesc, true);
    }
    mma_commit(&bar);
    if (!mbar_wait_bounded(&bar, 0, kWaitLimitNs) && err) atomicCAS(err, 0u, static_cast<unsigned>(kDevMmaTimeout));
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  if ((threadIdx.x >> 5) == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
}

}  // namespace tc

size_t gemm_tc_workspace_bytes(int m, int n, int d, int sm_count) {
  const tc::Plan p = tc::plan(m, n, d, sm_count);
  if (p.splits <= 1) return 256;
  return 256 + static_cast<size_t>(p.splits) * m * d * sizeof(float);
}

// Tensor-core path: m >= 16, n % 128 == 0, group 64, 16-byte aligned
// operands.  Returns MLI_ERR_UNSUPPORTED (without launching) otherwise.
int gemm_w8a8_tc(float* y, const int8_t* xq, const float* xs, const int8_t* w_q, const float* w_s,
                 int m, int n, int d, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (m < 16 || n % tc::kChunk != 0 || !aligned(xq, 16) || !aligned(w_q, 16))
    return set_status(MLI_ERR_UNSUPPORTED);
  cudaError_t err = cudaSuccess;
  const DeviceInfo& dev = current_device(&err);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  {
    const mli_gemm_op op = {y, xq, xs, w_q, w_s, n, d};
    const int pr = tc::launch_persistent(&op, 1, m, dev, stream);
    if (pr != -1) return pr;
  }
  const bool have_ws = workspace != nullptr &&
                       workspace_bytes >= gemm_tc_workspace_bytes(m, n, d, dev.sm_count);
  const tc::Plan p = tc::choose(m, n, d, dev, have_ws);
  CUtensorMap mw, mx;
  if (!tc::make_map(&mw, w_q, d, n, tc::kBM) || !tc::make_map(&mx, xq, m, n, p.bn))
    return set_status(MLI_ERR_UNSUPPORTED);
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
  a.cluster = p.cluster;
  a.err = device_error_word();
  const bool via_workspace = p.splits > 1 && p.cluster == 1;
  if (via_workspace) a.partial = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + 256);
  a.vec4 = d % 4 == 0 && aligned(y, 16) && (!via_workspace || aligned(a.partial, 16));
  const int grid = p.tiles_m * p.tiles_n * p.splits;
  switch (p.bn) {
    case 16: err = tc::launch_bn<16>(mw, mx, a, grid, stream); break;
    case 32: err = tc::launch_bn<32>(mw, mx, a, grid, stream); break;
    case 64: err = tc::launch_bn<64>(mw, mx, a, grid, stream); break;
    default: err = tc::launch_bn<128>(mw, mx, a, grid, stream); break;
  }
  if (err != cudaSuccess || !via_workspace) return check_cuda(err);
  const size_t per_block = static_cast<size_t>(tc::kReduceThreads) * tc::kReduceElems;
  const size_t md = static_cast<size_t>(m) * d;
  const unsigned blocks = static_cast<unsigned>((md + per_block - 1) / per_block);
  return check_cuda(launch(tc::splitk_reduce_kernel, dim3(blocks), dim3(tc::kReduceThreads), 0, stream, true,
                           y, static_cast<const float*>(a.partial), xs, p.splits, m, d, a.vec4));
}

// Several independent GEMMs of m tokens in one launch (mli_gemm_w8a8_group).
// Ops run largest K first; every op splits K the same number of ways (a
// cluster of that many blocks per tile): the fewest splits that keep one
// block's K range within three quarters of the average work per SM.
int gemm_w8a8_tc_group(const mli_gemm_op* ops, int count, int m, cudaStream_t stream) {
  cudaError_t err = cudaSuccess;
  const DeviceInfo& dev = current_device(&err);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  {
    const int pr = tc::launch_persistent(ops, count, m, dev, stream);
    if (pr != -1) return pr;
  }
  int order[tc::kMaxGroupOps];
  for (int i = 0; i < count; ++i) order[i] = i;
  for (int i = 1; i < count; ++i)  // insertion sort, largest n first (stable)
    for (int j = i; j > 0 && ops[order[j]].n > ops[order[j - 1]].n; --j) {
      const int t = order[j];
      order[j] = order[j - 1];
      order[j - 1] = t;
    }
  tc::Plan plans[tc::kMaxGroupOps];
  long long work = 0;
  int max_chunks = 0, min_chunks = 1 << 30;
  for (int i = 0; i < count; ++i) {
    plans[i] = tc::plan(m, ops[i].n, ops[i].d, dev.sm_count);
    work += static_cast<long long>(plans[i].tiles_m) * plans[i].tiles_n * plans[i].chunks;
    max_chunks = plans[i].chunks > max_chunks ? plans[i].chunks : max_chunks;
    min_chunks = plans[i].chunks < min_chunks ? plans[i].chunks : min_chunks;
  }
  const double per_sm = static_cast<double>(work) / dev.sm_count;
  int splits = 1;
  while (splits < 4 && min_chunks / (2 * splits) >= 2 &&
         static_cast<double>((max_chunks + splits - 1) / splits) > 0.75 * per_sm)
    splits *= 2;
  tc::GroupArgs g = {};
  g.count = count;
  int blocks = 0;
  unsigned int* err_word = device_error_word();
  for (int k = 0; k < count; ++k) {
    const mli_gemm_op& op = ops[order[k]];
    const tc::Plan& p = plans[order[k]];
    if (!tc::make_map(&g.mw[k], op.w_q, op.d, op.n, tc::kBM) || !tc::make_map(&g.mx[k], op.xq, m, op.n, p.bn))
      return set_status(MLI_ERR_UNSUPPORTED);
    tc::Args& a = g.op[k];
    a.y = op.y;
    a.xs = op.xs;
    a.ws = op.w_s;
    a.m = m;
    a.n = op.n;
    a.d = op.d;
    a.G = op.n / 64;
    a.bn = p.bn;
    a.tiles_m = p.tiles_m;
    a.tiles_n = p.tiles_n;
    a.splits = splits;
    a.chunks = p.chunks;
    a.cluster = splits;
    a.err = err_word;
    a.vec4 = op.d % 4 == 0 && aligned(op.y, 16);
    g.base[k] = blocks;
    blocks += p.tiles_m * p.tiles_n * splits;
  }
  g.base[count] = blocks;
  switch (plans[0].bn) {
    case 16: err = tc::launch_group_bn<16>(g, blocks, splits, stream); break;
    case 32: err = tc::launch_group_bn<32>(g, blocks, splits, stream); break;
    case 64: err = tc::launch_group_bn<64>(g, blocks, splits, stream); break;
    default: err = tc::launch_group_bn<128>(g, blocks, splits, stream); break;
  }
  return check_cuda(err);
}

}  // namespace mli

extern "C" int mli_gemm_w8a8_group(const mli_gemm_op* ops, int count, int m, int group_size, void* stream) {
  using namespace mli;
  if (!ops || count <= 0 || m <= 0 || group_size <= 0) return set_status(MLI_ERR_INVALID_ARG);
  if (count > tc::kMaxGroupOps) return set_status(MLI_ERR_UNSUPPORTED);
  for (int i = 0; i < count; ++i) {
    const mli_gemm_op& op = ops[i];
    if (!op.y || !op.xq || !op.xs || !op.w_q || !op.w_s || op.n <= 0 || op.d <= 0)
      return set_status(MLI_ERR_INVALID_ARG);
  }
  // the tensor-core shapes only; anything else is refused rather than run elsewhere
  if (group_size != 64 || m < 16) return set_status(MLI_ERR_UNSUPPORTED);
  for (int i = 0; i < count; ++i)
    if (ops[i].n % tc::kChunk != 0 || !aligned(ops[i].xq, 16) || !aligned(ops[i].w_q, 16))
      return set_status(MLI_ERR_UNSUPPORTED);
  return gemm_w8a8_tc_group(ops, count, m, static_cast<cudaStream_t>(stream));
}

extern "C" int mli_debug_int8_mma_peak(int n, int iters, int ctas, void* stream) {
  using namespace mli;
  if ((n != 64 && n != 128 && n != 256) || iters <= 0 || ctas <= 0) return set_status(MLI_ERR_INVALID_ARG);
  // more than half of an SM's shared memory: one CTA per SM, so no CTA waits
  // for another's tensor memory
  const size_t need = 1024u + tc::kStageA + static_cast<size_t>(n) * tc::kChunk;
  const size_t smem = need > 120u * 1024u ? need : 120u * 1024u;
  const void* fn = n == 256 ? reinterpret_cast<const void*>(tc::mma_peak_kernel<256>)
                   : n == 128 ? reinterpret_cast<const void*>(tc::mma_peak_kernel<128>)
                              : reinterpret_cast<const void*>(tc::mma_peak_kernel<64>);
  cudaError_t e = ensure_dynamic_smem(fn, smem);
  if (e != cudaSuccess) return check_cuda(e);
  unsigned int* err = device_error_word();
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (n) {
    case 256: e = launch(tc::mma_peak_kernel<256>, dim3(ctas), dim3(128), smem, st, false, iters, err); break;
    case 128: e = launch(tc::mma_peak_kernel<128>, dim3(ctas), dim3(128), smem, st, false, iters, err); break;
    default: e = launch(tc::mma_peak_kernel<64>, dim3(ctas), dim3(128), smem, st, false, iters, err); break;
  }
  return check_cuda(e);
}

extern "C" int mli_debug_plan_gemm_group(const mli_gemm_op* ops, int count, int m, int* out) {
  using namespace mli;
  if (!ops || !out || count < 1 || count > MLI_GEMM_GROUP_MAX || m <= 0) return set_status(MLI_ERR_INVALID_ARG);
  for (int i = 0; i < count; ++i)
    if (ops[i].n <= 0 || ops[i].d <= 0) return set_status(MLI_ERR_INVALID_ARG);
  cudaError_t err = cudaSuccess;
  const DeviceInfo& dev = current_device(&err);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  const tc::PChoice ch = tc::persistent_plan(ops, count, m, dev, nullptr);
  out[0] = ch.use ? 1 : 0;
  out[1] = ch.ctas;
  out[2] = ch.units;
  out[3] = static_cast<int>(ch.makespan);
  out[4] = static_cast<int>(ch.total);
  return set_status(MLI_OK);
}

extern "C" int mli_debug_plan_gemm(int m, int n, int d, size_t workspace_bytes, int* out) {
  using namespace mli;
  if (!out || m <= 0 || n <= 0 || d <= 0) return set_status(MLI_ERR_INVALID_ARG);
  if (m < 16 || n % tc::kChunk != 0) return set_status(MLI_ERR_UNSUPPORTED);
  cudaError_t err = cudaSuccess;
  const DeviceInfo& dev = current_device(&err);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  const bool have_ws = workspace_bytes >= gemm_tc_workspace_bytes(m, n, d, dev.sm_count);
  const tc::Plan p = tc::choose(m, n, d, dev, have_ws);
  out[0] = p.bn;
  out[1] = p.tiles_m * p.tiles_n;
  out[2] = p.splits;
  out[3] = p.cluster;
  out[4] = p.splits > 1 && p.cluster == 1;
  return set_status(MLI_OK);
}

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
