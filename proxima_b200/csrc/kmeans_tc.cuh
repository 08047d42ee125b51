// kmeans_tc.cuh — K7a: nearest-centroid screening for k-means on tcgen05
// tensor cores (kind::tf32). This kernel never decides an assignment; it
// narrows, for every point p, the set of centroids that can still be the
// reference's exact winner (crates/proxima-quantize/src/kmeans.rs:200-212,
// sequential f32 sum, strict '<', ties to the lower index).
//
// With a(c) = ||c||^2 - 2 p.c (TF32 product, FP32 accumulate, FP32 norms):
//   MIN pass   writes min_c a(c) per point;
//   CAND pass  every centroid that can still win (or tie) the exact argmin
//              satisfies a(c) <= min(T_prior, T(m)), where m is the smallest
//              score seen so far and T(m) = A (B + m) + Cc (A uniform; B, Cc
//              and T_prior per point, all rounded up by the host-side bound).
//              The kernel writes those centroids in ascending order (at most
//              CMAX) and their true count; a count above CMAX sends the point
//              to an exact rescan.
//
// Structure: one CTA per 256 points and all centroids.
//   warp 0    TMA producer (128-byte swizzle): the point tile
//             once, then 256-centroid tiles through a ring of K-block stages;
//   warp 1    TMEM allocator and MMA issuer: M=128, N=256, K=8 per
//             tcgen05.mma kind::tf32, one 256-column accumulator per point half;
//   warps 2-9 one thread per point: tcgen05.ld 32 columns at a time.
// When the ring holds a whole centroid tile (stages >= K blocks) the two
// halves are staggered so the MMAs of one half overlap the other half's
// epilogue; otherwise both halves advance together per K block.
// Every wait is bounded; a timeout sets the device error word and the kernel
// drains its copies and returns.
#pragma once
#include "common.cuh"
#include "sm100.cuh"

namespace pxc {
namespace km_tc {

constexpr int BM = 256;
constexpr int UM = 128;
constexpr int BN = 256;
constexpr int KB_BYTES = 128;  // 32 floats per K block (one 128-byte swizzle row)
constexpr int KB_FLOATS = 32;
constexpr int UMMA_K_BYTES = 32;  // 8 tf32 per tcgen05.mma
constexpr int A_BLOCK = BM * KB_BYTES;  // 32 KiB
constexpr int B_BLOCK = BN * KB_BYTES;  // 32 KiB
constexpr int NUM_EPI_WARPS = 8;
constexpr int NUM_THREADS = 64 + 32 * NUM_EPI_WARPS;
constexpr int MAX_KBLOCKS = 4;  // dim <= 128
constexpr int CMAX = 8;         // candidates kept per point
constexpr size_t SMEM_LIMIT = 232448 - 1024;  // 227 KiB opt-in less the 1 KiB-aligned static block

struct Params {
  const float* cnorm;    // ||c||^2 per centroid, +inf for the padding up to a multiple of 256
  const float4* bound;   // CAND: per point x = T_prior (+inf when none), y = B, z = Cc
  float A;               // CAND: uniform slope of T(m)
  float* out_min;        // MIN: per-point min a(c)
  uint32_t* out_cnt;     // CAND: per-point candidate count (may exceed CMAX)
  uint32_t* out_cand;    // CAND: [point][CMAX] centroid indices, ascending
  uint32_t* status;      // device error word [code, block]
  uint32_t npoints;
  uint32_t kblocks;
  uint32_t ntiles;       // centroid tiles of 256
  uint32_t stages;
  uint64_t wait_ns;
};

__host__ inline size_t smem_bytes(uint32_t kblocks, uint32_t stages) {
  return 1024 + (size_t)kblocks * A_BLOCK + (size_t)stages * B_BLOCK + (2 * stages + 8) * 8 + 16;
}
__host__ inline uint32_t pick_stages(uint32_t kblocks) {
  uint32_t s = 8;
  while (s > 2 && smem_bytes(kblocks, s) > SMEM_LIMIT) --s;
  return s;
}

// Instruction descriptor for kind::tf32: tf32 x tf32 -> f32, both K-major
// (PTX ISA instruction-descriptor table; CUTLASS UMMA::InstrDescriptor).
__host__ __device__ constexpr uint32_t idesc_tf32_f32(uint32_t m, uint32_t n) {
  return (1u << 4)     // D format: f32
         | (2u << 7)   // A: tf32
         | (2u << 10)  // B: tf32
         | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void record_failure(uint32_t* status, uint32_t code) {
  if (atomicCAS(status, 0u, code) == 0u) atomicExch(status + 1, blockIdx.x);
}

template <bool MIN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    screen_kernel(const __grid_constant__ CUtensorMap tmap_p, const __grid_constant__ CUtensorMap tmap_c,
                  const Params p) {
  using namespace sm100;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t kblocks = p.kblocks, stages = p.stages, ntiles = p.ntiles;
  const bool stagger = stages >= kblocks;
  unsigned char* sA = smem;
  unsigned char* sB = smem + (size_t)kblocks * A_BLOCK;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + (size_t)stages * B_BLOCK);
  uint64_t* full = bars;
  uint64_t* empty = bars + stages;
  uint64_t* acc_full = bars + 2 * stages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* a_full = acc_empty + 2;
  uint64_t* mma_done = a_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  __shared__ volatile uint32_t failed;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ptile = blockIdx.x;

  if (warp == 1) {
    tmem_alloc<512>(tmem_slot);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    failed = 0;
    for (uint32_t s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int m = 0; m < 2; ++m) {
      mbar_init(&acc_full[m], 1);
      mbar_init(&acc_empty[m], 4 * 32);
    }
    mbar_init(a_full, 1);
    mbar_init(mma_done, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmap_p);
    tma_prefetch_desc(&tmap_c);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      mbar_arrive_expect_tx(a_full, kblocks * A_BLOCK);
      for (uint32_t kb = 0; kb < kblocks; ++kb)
        tma_load_2d(sA + (size_t)kb * A_BLOCK, &tmap_p, a_full, kb * KB_FLOATS, ptile * BM);
    }
    __syncwarp();
    uint32_t it = 0;
    bool ok = true;
    for (uint32_t t = 0; t < ntiles && ok; ++t) {
      for (uint32_t kb = 0; kb < kblocks; ++kb, ++it) {
        const uint32_t s = it % stages, ph = (it / stages) & 1;
        const bool fl = failed;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&empty[s], ph ^ 1, p.wait_ns) && !fl)) {
          if (lane == 0) record_failure(p.status, DEV_TIMEOUT_EMPTY);
          failed = 1;
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[s], B_BLOCK);
          tma_load_2d(sB + (size_t)s * B_BLOCK, &tmap_c, &full[s], kb * KB_FLOATS, t * BN);
        }
        __syncwarp();
      }
    }
    // Drain: no copy may land after the CTA exits.
    const uint32_t first = it > stages ? it - stages : 0;
    for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % stages], (j / stages) & 1, p.wait_ns);
    mbar_wait(a_full, 0, p.wait_ns);
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = idesc_tf32_f32(UM, BN);
    bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(a_full, 0, p.wait_ns));
    if (!ok) {
      if (lane == 0) record_failure(p.status, DEV_TIMEOUT_FULL);
      failed = 1;
    }
    tc_fence_after();
    const uint32_t a_addr = smem_u32(sA), b_addr = smem_u32(sB);
    auto wait_or_fail = [&](uint64_t* bar, uint32_t parity, uint32_t code) -> bool {
      const bool fl = failed;
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(bar, parity, p.wait_ns) && !fl)) {
        if (lane == 0) record_failure(p.status, code);
        failed = 1;
        return false;
      }
      tc_fence_after();
      return true;
    };
    auto issue = [&](uint32_t m, uint32_t kb, uint32_t s) {
      if (lane == 0) {
        const uint64_t bdesc = smem_desc_k_sw128(b_addr + s * B_BLOCK);
        const uint64_t adesc = smem_desc_k_sw128(a_addr + kb * A_BLOCK + m * (UM * KB_BYTES));
#pragma unroll
        for (uint32_t k = 0; k < KB_BYTES / UMMA_K_BYTES; ++k)
          mma_tf32(tmem_base + m * BN, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0);
      }
      __syncwarp();
    };
    for (uint32_t t = 0; t < ntiles && ok; ++t) {
      const uint32_t it0 = t * kblocks;
      if (stagger) {
        for (uint32_t m = 0; m < 2 && ok; ++m) {
          if (!(ok = wait_or_fail(&acc_empty[m], (t & 1) ^ 1, DEV_TIMEOUT_ACC))) break;
          for (uint32_t kb = 0; kb < kblocks; ++kb) {
            const uint32_t it = it0 + kb, s = it % stages, ph = (it / stages) & 1;
            if (m == 0 && !(ok = wait_or_fail(&full[s], ph, DEV_TIMEOUT_FULL))) break;
            issue(m, kb, s);
          }
          if (!ok) break;
          if (lane == 0) mma_commit(&acc_full[m]);
          __syncwarp();
        }
        if (!ok) break;
        if (lane == 0)
          for (uint32_t kb = 0; kb < kblocks; ++kb) mma_commit(&empty[(it0 + kb) % stages]);
        __syncwarp();
      } else {
        if (!(ok = wait_or_fail(&acc_empty[0], (t & 1) ^ 1, DEV_TIMEOUT_ACC))) break;
        if (!(ok = wait_or_fail(&acc_empty[1], (t & 1) ^ 1, DEV_TIMEOUT_ACC))) break;
        for (uint32_t kb = 0; kb < kblocks; ++kb) {
          const uint32_t it = it0 + kb, s = it % stages, ph = (it / stages) & 1;
          if (!(ok = wait_or_fail(&full[s], ph, DEV_TIMEOUT_FULL))) break;
          issue(0, kb, s);
          issue(1, kb, s);
          if (lane == 0) mma_commit(&empty[s]);
          __syncwarp();
        }
        if (!ok) break;
        if (lane == 0) {
          mma_commit(&acc_full[0]);
          mma_commit(&acc_full[1]);
        }
        __syncwarp();
      }
    }
    if (lane == 0) mma_commit(mma_done);
    __syncwarp();
    mbar_wait(mma_done, 0, p.wait_ns);
  } else {
    // ---------------- epilogue: one thread per point ----------------
    const uint32_t ew = warp - 2, quarter = warp & 3, half = ew >> 2;
    const uint32_t row = half * UM + quarter * 32 + lane;
    const uint32_t pidx = ptile * BM + row;
    const bool valid = pidx < p.npoints;
    const float inf = __int_as_float(0x7f800000);
    float4 bnd = make_float4(-inf, 0.0f, 0.0f, 0.0f);
    if (!MIN && valid) bnd = p.bound[pidx];
    const float thr_prior = bnd.x, B = bnd.y, Cc = bnd.z, A = p.A;
    // upper bound on every possible winner's score given the running minimum m
    auto t_of = [&](float m) {
      const float t = fmaf(A, fmaxf(0.0f, B + m), Cc);
      return t + 0x1p-18f * (B + fabsf(m) + fabsf(Cc)) + 0x1p-100f;
    };
    float run_min = inf;
    uint32_t cnt = 0;
    uint32_t* my_cand = MIN ? nullptr : p.out_cand + (size_t)pidx * CMAX;
    for (uint32_t t = 0; t < ntiles; ++t) {
      const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&acc_full[half], t & 1, p.wait_ns) && !failed);
      if (!ok) {
        if (lane == 0) record_failure(p.status, DEV_TIMEOUT_ACC);
        failed = 1;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((quarter * 32) << 16) + half * BN;
      const float4* nrm = reinterpret_cast<const float4*>(p.cnorm + (size_t)t * BN);
      // One 32-column chunk: scores, chunk minimum and, in the CAND pass, the
      // (rare) centroids under the threshold.
      auto process = [&](uint32_t(&v)[32], const float4(&n4)[8], uint32_t c) {
        float cmin = inf;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float nn[4] = {n4[q].x, n4[q].y, n4[q].z, n4[q].w};
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const float a = fmaf(-2.0f, __uint_as_float(v[4 * q + r]), nn[r]);
            v[4 * q + r] = __float_as_uint(a);
            cmin = fminf(cmin, a);
          }
        }
        run_min = fminf(run_min, cmin);
        if (MIN) return;
        const float thr = valid ? fminf(thr_prior, t_of(run_min)) : -inf;
        const bool hit = cmin <= thr;  // some score of the chunk is under the threshold
        if (__any_sync(0xFFFFFFFFu, hit) && hit) {
          uint32_t m = 0;
#pragma unroll
          for (int j = 0; j < 32; ++j) m |= (__uint_as_float(v[j]) <= thr ? 1u : 0u) << j;
          const uint32_t base = t * BN + c * 32;
          while (m) {
            const int j = __ffs(m) - 1;
            m &= m - 1;
            if (cnt < CMAX) my_cand[cnt] = base + j;
            ++cnt;
          }
        }
      };
      // TMEM loads and norm loads double-buffered: the next chunk's data is in
      // flight while this one is processed (tcgen05.wait::ld waits for both).
      uint32_t va[32], vb[32];
      float4 na[8], nb[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) na[q] = __ldg(nrm + q);
      tmem_ld_32x32b_x32(taddr, va);
      tmem_ld_wait();
#pragma unroll 1
      for (uint32_t c = 0; c < BN / 32; c += 2) {
        tmem_ld_32x32b_x32(taddr + (c + 1) * 32, vb);
#pragma unroll
        for (int q = 0; q < 8; ++q) nb[q] = __ldg(nrm + (c + 1) * 8 + q);
        process(va, na, c);
        tmem_ld_wait();
        if (c + 2 < BN / 32) {
          tmem_ld_32x32b_x32(taddr + (c + 2) * 32, va);
#pragma unroll
          for (int q = 0; q < 8; ++q) na[q] = __ldg(nrm + (c + 2) * 8 + q);
        }
        process(vb, nb, c + 1);
        tmem_ld_wait();
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[half]);
    }
    if (valid) {
      if (MIN)
        p.out_min[pidx] = run_min;
      else
        p.out_cnt[pidx] = failed ? 0xFFFFFFFFu : cnt;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc<512>(tmem_base);
}

}  // namespace km_tc
}  // namespace pxc
