// mli_common.cuh -- shared device helpers for the B200 (sm_100a) INT8 group-64
// linear kernels: PTX wrappers for bulk async copies, mbarriers, programmatic
// dependent launch, packed fp32x2 arithmetic and int8 -> fp32 conversion.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mli_gemv.h"

namespace mli {

// ---------------------------------------------------------------------------
// Device-side error word.  Kernels that give up on a bounded wait record a
// code here and return; the host reads it with mli_device_error().
// ---------------------------------------------------------------------------
enum DeviceError : unsigned int {
  kDevOk = 0,
  kDevStageTimeout = 1,  // bulk copy of the activation vector never landed
  kDevMmaTimeout = 2,    // tensor-core pipeline barrier never completed
  kDevPeerTimeout = 3,   // rows of a row-sharded step never arrived from a rank
  kDevChainTimeout = 4,  // a chained GEMV's inputs were never completed
  kDevScaleRange = 5,    // a group scale outside the batched tensor-core path's exact range
};
#ifndef MLI_SEPARATE_DEVICE_MODULE
extern __device__ unsigned int g_device_error;
#endif

// Row-sharded layers (gemv_g64.cu, rowshard.cu): at most this many ranks and
// CTAs per rank.  A rank's peer block holds its logits as 8-byte words
// [2][d_total] (the half is the step's parity), then, at the next 16-byte
// boundary, one 8-byte partial word per CTA of every rank,
// [2][kMaxPeers][kMaxRankCtas].  Every word carries the tag of the step that
// wrote it, so a reader knows a word has arrived by the word alone:
//   logits word:  low 32 bits the fp32 value, high 32 bits the tag;
//   partial word: low 32 bits the CTA's maximum (fp32), high 32 bits
//                 (first index << 12) | tag  (indices below 2^20).
// Tags cycle 1 .. kRowTagPeriod; zeroed memory (tag 0) never matches.
constexpr int kMaxPeers = 8;
constexpr int kMaxRankCtas = 512;
constexpr unsigned kRowTagPeriod = 4095;
constexpr int kMaxRowshardRows = 1 << 20;

__host__ __device__ __forceinline__ unsigned rowshard_tag(unsigned step) {
  return step % kRowTagPeriod + 1;
}
__host__ __device__ __forceinline__ unsigned long long* rowshard_partials(unsigned long long* logits,
                                                                         int d_total) {
  return logits + ((static_cast<size_t>(d_total) * 2u + 1u) & ~static_cast<size_t>(1));
}
__host__ __device__ __forceinline__ const unsigned long long* rowshard_partials(const unsigned long long* logits,
                                                                               int d_total) {
  return rowshard_partials(const_cast<unsigned long long*>(logits), d_total);
}
__host__ __device__ constexpr size_t rowshard_block_bytes(int d_total) {
  return 256 + ((static_cast<size_t>(d_total) * 2u + 1u) & ~static_cast<size_t>(1)) * 8u +
         8u * 2 * kMaxPeers * kMaxRankCtas;
}

// System-scope relaxed 8-byte accesses of tagged words (single-copy atomic:
// a reader sees a value together with its tag).
__device__ __forceinline__ void st_relaxed_sys_b64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_b64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long tag_word(uint32_t lo, uint32_t hi) {
  return (static_cast<unsigned long long>(hi) << 32) | lo;
}

#ifndef MLI_SEPARATE_DEVICE_MODULE
__device__ __forceinline__ void record_device_error(unsigned int code) {
  atomicCAS(&g_device_error, 0u, code);
}
#endif

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched with
// cudaLaunchAttributeProgrammaticStreamSerialization may start while the
// previous kernel in the stream drains; it reads nothing that kernel wrote
// before griddep_wait().  Both are no-ops for kernels launched without it.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// mbarrier + 1-D bulk copy (TMA engine, no tensor map needed).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

// Orders this thread's earlier generic-proxy accesses of shared memory
// before later async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Global -> shared bulk copy of `bytes` (multiple of 16, both addresses
// 16-byte aligned), completion signalled on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_copy_g2s(void* dst_smem, const void* src,
                                              uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], "
      "[%1], %2, [%3];" ::"r"(smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Asks the TMA engine to bring `bytes` (multiple of 16; 16-byte aligned
// source) into L2 without a destination or completion: a later bulk copy of
// the same bytes then reads L2 instead of HBM.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after `limit_ns` of global time and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar,
                                                  uint32_t parity,
                                                  uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
  return true;
}

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// ---------------------------------------------------------------------------
// Streaming loads: weights are read exactly once, so bypass L1.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ldg_f4(const float* p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ float ldg_f1(const float* p) {
  float v;
  asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

// ---------------------------------------------------------------------------
// Packed fp32x2 arithmetic (sm_100a): one instruction for two lanes of fp32.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rc, rd;\n"
      "mov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nmov.b64 rc, {%6, %7};\n"
      "fma.rn.f32x2 rd, ra, rb, rc;\nmov.b64 {%0, %1}, rd;\n}\n"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rd;\n"
      "mov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
      "mul.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}\n"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rd;\n"
      "mov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
      "add.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}\n"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// ---------------------------------------------------------------------------
// Exact int8 -> fp32.  A byte b (signed) is flipped to b + 128 (unsigned) and
// placed under the exponent of 2^23, giving the float 2^23 + b + 128 exactly;
// subtracting 2^23 + 128 recovers b.  One byte-permute per value plus one
// packed subtract per pair replaces the slower integer-to-float conversion.
// ---------------------------------------------------------------------------
constexpr float kI8Magic = 8388736.0f;  // 2^23 + 128

// Returns the magic-biased floats of bytes 2*h and 2*h+1 of `u_flipped`
// (a word already XORed with 0x80808080).
template <int kHalf>
__device__ __forceinline__ float2 biased_pair(uint32_t u_flipped) {
  float2 r;
  r.x = __uint_as_float(__byte_perm(u_flipped, 0x4B000000u, 0x7540 + 2 * kHalf));
  r.y = __uint_as_float(__byte_perm(u_flipped, 0x4B000000u, 0x7541 + 2 * kHalf));
  return r;
}

// Named barrier 1 over the first `kCount` threads of the CTA (the consumer
// warps of a warp-specialised kernel; the producer warp never joins it).
template <int kCount>
__device__ __forceinline__ void named_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kCount) : "memory");
}
// Same barrier, returning whether `pred` held on any participating thread.
template <int kCount>
__device__ __forceinline__ bool named_sync_or(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n.reg .pred p, q;\n"
      "setp.ne.u32 p, %1, 0;\n"
      "bar.red.or.pred q, 1, %2, p;\n"
      "selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "n"(kCount)
      : "memory");
  return r != 0;
}

// First-maximum rule of the reference's host scan (`if (logits[i] > max_val)`
// starting from max_val = logits[0]): a larger value wins, equal values keep
// the smaller index, -0.0 and +0.0 are equal, a NaN never wins (every
// comparison with it is false) -- and a NaN in x[0] makes the answer 0.
__device__ __forceinline__ void argmax_combine(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

// Completes a row-sharded step on kT threads of one CTA: polls every rank's
// CTA partial words of this step (tag `tag`, half `parity` of this rank's
// block), reduces them to the first maximum of the full logits (the
// reference's host argmax, src/main_cuda.cpp:96-98), and returns it on every
// thread -- or -1 if a word did not arrive within timeout_ns.  Each thread
// loads all of its words at once and reloads only the missing ones, so a step
// costs one round trip per retry, not one per word.  `red_v` / `red_i` hold
// kT / 32 entries; `s_int` is one shared int.
template <int kT>
__device__ __forceinline__ long long rowshard_poll_argmax(const unsigned long long* logits, int d_total,
                                                          unsigned parity, unsigned tag, int world,
                                                          const int* shard_ctas, unsigned long long timeout_ns,
                                                          float* red_v, int* red_i, int* s_int) {
  constexpr int kPer = (kMaxPeers * kMaxRankCtas + kT - 1) / kT;
  const unsigned long long* parts = rowshard_partials(logits, d_total) +
                                    static_cast<size_t>(parity) * kMaxPeers * kMaxRankCtas;
  int start[kMaxPeers + 1];
  start[0] = 0;
#pragma unroll
  for (int r = 0; r < kMaxPeers; ++r) start[r + 1] = start[r] + (r < world ? shard_ctas[r] : 0);
  const int total = start[kMaxPeers];
  // this thread's words: flat indices threadIdx.x + k kT, k < kPer
  unsigned pending = 0;
  int slot[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int f = static_cast<int>(threadIdx.x) + k * kT;
    slot[k] = 0;
    if (f < total) {
      int r = 0;
#pragma unroll
      for (int q = 1; q < kMaxPeers; ++q) r += f >= start[q] ? 1 : 0;
      slot[k] = r * kMaxRankCtas + (f - start[r]);
      pending |= 1u << k;
    }
  }
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  bool fail = false;
  const uint64_t t0 = global_timer_ns();
  unsigned ns = 32;
  while (pending != 0) {
    unsigned long long w[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k)
      if ((pending >> k) & 1u) w[k] = ld_relaxed_sys_b64(parts + slot[k]);
#pragma unroll
    for (int k = 0; k < kPer; ++k)
      if (((pending >> k) & 1u) && (static_cast<unsigned>(w[k] >> 32) & 0xfffu) == tag) {
        argmax_combine(bv, bi, __uint_as_float(static_cast<unsigned>(w[k])), static_cast<int>(w[k] >> 44));
        pending &= ~(1u << k);
      }
    if (pending == 0) break;
    if (global_timer_ns() - t0 > timeout_ns) {
      fail = true;
      break;
    }
    __nanosleep(ns);
    ns = ns < 256 ? 2 * ns : 256;
  }
  // the reference's scan starts from x[0]: its value decides a NaN start
  float x0 = 0.f;
  if (threadIdx.x == 0 && !fail) {
    const unsigned long long* w0 = logits + static_cast<size_t>(parity) * d_total;
    unsigned long long w = ld_relaxed_sys_b64(w0);
    while (static_cast<unsigned>(w >> 32) != tag) {
      if (global_timer_ns() - t0 > timeout_ns) {
        fail = true;
        break;
      }
      __nanosleep(64);
      w = ld_relaxed_sys_b64(w0);
    }
    x0 = __uint_as_float(static_cast<unsigned>(w));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    argmax_combine(bv, bi, ov, oi);
  }
  if (threadIdx.x == 0) *s_int = 0;
  __syncthreads();
  if (fail) atomicExch(s_int, 1);
  if ((threadIdx.x & 31) == 0) {
    red_v[threadIdx.x >> 5] = bv;
    red_i[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  const bool failed = *s_int != 0;
  bv = red_v[0];
  bi = red_i[0];
#pragma unroll
  for (int w = 1; w < kT / 32; ++w) argmax_combine(bv, bi, red_v[w], red_i[w]);
  __syncthreads();
  if (threadIdx.x == 0) *s_int = (bi == 0x7fffffff || x0 != x0) ? 0 : bi;
  __syncthreads();
  const long long res = failed ? -1 : *s_int;
  __syncthreads();
  return res;
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}
// Sums RB per-lane values (one per row) across the warp at once: a
// transposed butterfly halves the rows held per lane at offsets 16, 8, ...
// and finishes with a plain butterfly.  Row r's total ends up in lane
// r * (32 / RB) (among others).  Every row is summed with the same tree as
// warp_sum -- pairs across lane bit 4 first, then bits 3, 2, 1, 0 -- so the
// result is bit-identical to warp_sum of that row alone.
template <int RB>
__device__ __forceinline__ float warp_sum_rows(const float (&v)[RB], int lane) {
  static_assert(RB == 1 || RB == 2 || RB == 4 || RB == 8, "RB must be 1, 2, 4 or 8");
  float cur[RB];
#pragma unroll
  for (int i = 0; i < RB; ++i) cur[i] = v[i];
  int off = 16;
#pragma unroll
  for (int width = RB; width > 1; width >>= 1, off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < width / 2; ++i) {
      const float keep = upper ? cur[i + width / 2] : cur[i];
      const float send = upper ? cur[i] : cur[i + width / 2];
      cur[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
#pragma unroll
  for (; off > 0; off >>= 1) cur[0] += __shfl_xor_sync(0xffffffffu, cur[0], off);
  return cur[0];
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

}  // namespace mli
