// Device helpers of the B200 sampler: order-preserving keys, the fixed exp of the weights,
// fixed-point arithmetic, mbarrier / bulk-copy (TMA) PTX wrappers and block-level scans.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "pagedbatch_b200.h"

namespace pb {

constexpr uint32_t KEY_NEG_INF = 0x007FFFFFu;  // key of -inf
constexpr uint32_t KEY_POS_INF = 0xFF800000u;  // key of +inf (NaN maps above it)

// Order-preserving key: NaN above everything (torch.argmax / topk treat NaN as the largest),
// -0 folded onto +0 (IEEE compares them equal, so argmax and the top-k mask tie them).
__device__ __forceinline__ uint32_t key_of(float x) {
  if (x != x) return 0xFFFFFFFFu;
  uint32_t b = (x == 0.0f) ? 0u : __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float value_of(uint32_t k) {
  uint32_t b = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(b);
}

// Weight of a key d = key - max <= 0: e^d by Cody-Waite reduction (ln2 split in two) and the
// degree-7 Taylor polynomial of e^r on |r| <= ln2/2, every step an explicitly rounded fp32
// operation so that the CPU restatement reproduces the same bits. Max error 0.94 ulp against
// libm's exp over every fp32 in [-87, 0]; 0 below -87 (no subnormal results).
__device__ __forceinline__ float exp_weight(float d) {
  if (!(d >= -87.0f)) return 0.0f;
  const float t = __fmul_rn(d, 0x1.715476p+0f);
  const float n = rintf(t);
  float r = __fmaf_rn(-n, 0x1.62e43p-1f, d);
  r = __fmaf_rn(-n, -0x1.05c61p-29f, r);
  float p = 0x1.a01a02p-13f;
  p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
  p = __fmaf_rn(p, r, 0x1.111112p-7f);
  p = __fmaf_rn(p, r, 0x1.555556p-5f);
  p = __fmaf_rn(p, r, 0x1.555556p-3f);
  p = __fmaf_rn(p, r, 0x1.0p-1f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = __float2int_rn(n);
  return __int_as_float(__float_as_int(p) + (ni << 23));
}

// Fixed-point weight q = floor(e^(key - max) * 2^40); sums over < 2^24 elements fit in 64 bits.
__device__ __forceinline__ uint64_t weight_q(float key, float m) {
  const float w = exp_weight(__fsub_rn(key, m));
  return __float2ull_rz(__fmul_rn(w, 0x1p40f));
}

// floor(p * z) for fp32 p in [0, 1) and z < 2^64, exact (128-bit product).
__device__ __forceinline__ uint64_t mul_floor(float p, uint64_t z) {
  const uint32_t b = __float_as_uint(p);
  const uint32_t e8 = (b >> 23) & 0xFF;
  uint64_t man = b & 0x7FFFFF;
  int shift;
  if (e8 == 0) {
    shift = 149;
  } else {
    man |= 0x800000;
    shift = 150 - (int)e8;
  }
  if (shift >= 128 || man == 0) return 0;
  const uint64_t lo = man * z;
  const uint64_t hi = __umul64hi(man, z);
  if (shift >= 64) return hi >> (shift - 64);
  return (lo >> shift) | (hi << (64 - shift));
}

// floor(u53 * z / 2^53) for u53 < 2^53.
__device__ __forceinline__ uint64_t scale_u53(uint64_t u53, uint64_t z) {
  const uint64_t lo = u53 * z;
  const uint64_t hi = __umul64hi(u53, z);
  return (lo >> 53) | (hi << 11);
}

// Composite sort key: descending order = key descending, index ascending.
__device__ __forceinline__ uint64_t compose(uint32_t key, uint32_t idx) {
  return ((uint64_t)key << 32) | (uint64_t)(0xFFFFFFFFu - idx);
}
__device__ __forceinline__ uint32_t comp_key(uint64_t c) { return (uint32_t)(c >> 32); }
__device__ __forceinline__ uint32_t comp_idx(uint64_t c) { return 0xFFFFFFFFu - (uint32_t)c; }

// ---- per-row draws ---------------------------------------------------------------------------

// Philox4x32-10 (Salmon, Moraes, Dror and Shaw, "Parallel random numbers: as easy as 1, 2, 3",
// SC 2011): ten rounds of two 32x32->64 multiplications on a 4-word counter, with a 2-word key
// bumped by the Weyl constants between rounds.
__host__ __device__ __forceinline__ void philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2],
                                                       uint32_t out[4]) {
  uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
  uint32_t k0 = key_in[0], k1 = key_in[1];
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0, hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
  }
  out[0] = c0;
  out[1] = c1;
  out[2] = c2;
  out[3] = c3;
}

// U53 of a PB_RNG_PHILOX row: key = the 64-bit seed, counter = (step, 0, 0, 0).
__host__ __device__ __forceinline__ uint64_t philox_u53(uint64_t seed, uint32_t step) {
  const uint32_t ctr[4] = {step, 0u, 0u, 0u}, key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  uint32_t o[4];
  philox4x32_10(ctr, key, o);
  return ((uint64_t)(o[0] >> 11) << 32) | o[1];
}

// A row's draw as U53 (the draw is U53 / 2^53): its host-drawn uniform, or the device draw.
__host__ __device__ __forceinline__ uint64_t row_u53(const pb_row_params& p) {
  if (p.rng & PB_RNG_PHILOX) {
    uint64_t seed;
    memcpy(&seed, &p.uniform, 8);
    return philox_u53(seed, p.rng & 0x7FFFFFFFu);
  }
  return (uint64_t)(p.uniform * 0x1p53);
}

// Whether a row's draw is usable: device draws always are; a host draw must lie in [0, 1).
__host__ __device__ __forceinline__ bool row_draw_ok(const pb_row_params& p) {
  return (p.rng & PB_RNG_PHILOX) || (p.uniform >= 0.0 && p.uniform < 1.0);
}

// ---- mbarrier + bulk copy (TMA engine, 1-D, no multicast) -------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

// Shared-memory fetch-add with acquire-release ordering at CTA scope; returns the old value.
// plain arrival (no transaction bytes): completes the phase of a count-1 barrier by itself
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(smem_addr(p)), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(100000u)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after `limit` polls (each poll suspends up to ~0.1 ms) and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int limit) {
  for (int i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Global -> this CTA's shared memory, `bytes` (multiple of 16, both addresses 16-byte aligned),
// completion signalled on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Stores to shared memory under a predicate, without a branch (a predicated-off store costs an
// issue slot and nothing else).
__device__ __forceinline__ void st_shared_v4_if(bool p, void* dst, uint4 v) {
  asm volatile(
      "{\n .reg .pred q;\n setp.ne.u32 q, %0, 0;\n @q st.shared.v4.u32 [%1], {%2, %3, %4, %5};\n}\n" ::"r"((uint32_t)p),
      "r"(smem_addr(dst)), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
      : "memory");
}
__device__ __forceinline__ void st_shared_u32_if(bool p, void* dst, uint32_t v) {
  asm volatile("{\n .reg .pred q;\n setp.ne.u32 q, %0, 0;\n @q st.shared.u32 [%1], %2;\n}\n" ::"r"((uint32_t)p),
               "r"(smem_addr(dst)), "r"(v)
               : "memory");
}

// ---- warp / block scans -------------------------------------------------------------------

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

template <typename T>
__device__ __forceinline__ T warp_incl_scan(T v) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T n = __shfl_up_sync(0xFFFFFFFFu, v, o);
    if ((threadIdx.x & 31) >= (unsigned)o) v += n;
  }
  return v;
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// Barrier of a thread group: B = 0 is the whole CTA (__syncthreads); B = 1 and B = 2 are named
// barrier 1 over the first 256 or 512 threads (warps 0-7 or 0-15): a group of warps (the consumer
// warps of the streaming kernel) whose CTA's other warps run their own loops and never reach it.
template <int B>
__device__ __forceinline__ void bsync() {
  if constexpr (B == 0) {
    __syncthreads();
  } else if constexpr (B == 1) {
    asm volatile("bar.sync 1, 256;" ::: "memory");
  } else {
    asm volatile("bar.sync 1, 512;" ::: "memory");
  }
}

// Barrier of the group that also returns whether any of its threads passed v != 0.
template <int B>
__device__ __forceinline__ bool bsync_or(bool v) {
  if constexpr (B == 0) {
    return __syncthreads_or(v) != 0;
  } else {
    uint32_t r;
    if constexpr (B == 1) {
      asm volatile(
          "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, 256, p;\n selp.u32 %0, 1, 0, q;\n}\n"
          : "=r"(r)
          : "r"((uint32_t)v)
          : "memory");
    } else {
      asm volatile(
          "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, 512, p;\n selp.u32 %0, 1, 0, q;\n}\n"
          : "=r"(r)
          : "r"((uint32_t)v)
          : "memory");
    }
    return r != 0;
  }
}

// Block-wide exclusive scan of one value per thread; `scratch` holds >= nwarps + 1 entries.
// Returns the exclusive prefix; *total receives the block total. Contains barriers of group B.
template <typename T, int NT, int B = 0>
__device__ __forceinline__ T block_excl_scan(T v, T* scratch, T* total) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T inc = warp_incl_scan(v);
  if (lane == 31) scratch[warp] = inc;
  bsync<B>();
  if (warp == 0) {
    T s = (lane < NW) ? scratch[lane] : T(0);
    T si = warp_incl_scan(s);
    if (lane < NW) scratch[lane] = si - s;
    if (lane == NW - 1) scratch[NW] = si;
  }
  bsync<B>();
  T r = scratch[warp] + inc - v;
  *total = scratch[NW];
  bsync<B>();
  return r;
}

}  // namespace pb
