// tcgen05 tensor-core BAT contraction (sm_100a) for the NTT / INTT steps.
//
// One launch computes, for a batch of limb-polynomials that share a plan,
//     S[m, n] = sum_{w, q} byte_q(A[m, w]) * T_n[w, q]          (exact int)
//     out     = epilogue(Barrett(sum_p S_p << 8p))
// where A is an (rows_m x kw) uint32 matrix per limb-polynomial read as
// (rows_m x 4kw) uint8, and B is the reference's BAT twiddle array
// re-laid out as (4*nout x 4*kw) uint8 with row j = 4n + p, column 4w + q.
// This is matmul_bat_einsum + BarrettContext.modular_reduction of
// ntt_mm.py:20-37,201-230 for one 3-step NTT stage.
//
// Kernel structure (persistent, one CTA per SM, 192 threads):
//   warp 0      TMA producer: A tile 128 x 128 B, B tile 256 x 128 B per stage,
//               SWIZZLE_128B, 4-stage ring (plain loads, no multicast).
//   warp 1      TMEM allocation (512 columns) and the single MMA-issuing thread:
//               tcgen05.mma.cta_group::1.kind::i8, M=128 N=256 K=32, u8 x u8 -> s32,
//               accumulating into one of two 256-column TMEM buffers.
//   warps 2..17 epilogue, four warps per TMEM lane quadrant (each takes a
//               quarter of the 256 accumulator columns): tcgen05.ld rows, byte
//               recombination, Barrett, optional twiddle multiply (twiddles
//               prefetched before the accumulator is ready) + Barrett, stores;
//               runs while the MMA fills the other accumulator.
// Every mbarrier wait is bounded (about two seconds of wall time); on expiry the
// kernel records an error code, stops issuing work, lets its copies and MMAs
// drain (again bounded), frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "internal.hpp"
#include "tc_ptx.cuh"

namespace cross {
namespace tc {

constexpr int BM = 128;            // rows per tile (TMEM lanes)
constexpr int BN = 256;            // MMA N per tile: 64 outputs x 4 byte-planes
constexpr int BKB = 128;           // K bytes per pipeline stage (4 MMAs of K = 32)
constexpr int STAGES = 4;
constexpr int A_STAGE = BM * BKB;  // 16 KiB
constexpr int B_STAGE = BN * BKB;  // 32 KiB
constexpr int EPI_WARPS = 16;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t TMEM_COLS = 512;

struct Smem {
  uint8_t a[STAGES][A_STAGE];
  uint8_t b[STAGES][B_STAGE];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  volatile int abort;
};
constexpr size_t SMEM_BYTES = sizeof(Smem) + 1024;

struct Args {
  uint32_t* out;
  int64_t out_ps, out_ss;          // words
  const uint16_t* limbs;           // slot -> plan limb
  int slots;
  int64_t polys;
  int rows_m, kw, nout;
  const ModC* mods;
  const VarC* varc;                // Montgomery / BAT-lazy constants per plan limb (variant plans)
  int* err;
  Epi e;                           // fused position-wise op (EpiOp)
};

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* tm, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];" ::
          "r"(saddr(dst)),
      "l"((uint64_t)tm), "r"(saddr(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          saddr(dst)),
      "l"((uint64_t)tm), "r"(saddr(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// K-major, SWIZZLE_128B shared-memory matrix descriptor: 8-row atoms of
// 1024 B (stride-byte-offset 1024), leading-byte-offset 16 (unused when
// swizzled), descriptor version 1, layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::i8: D = S32 (bits 4-5 = 2), A = B = unsigned
// 8-bit (0), both K-major, N >> 3 in bits 17-22, M >> 4 in bits 24-28.
constexpr uint32_t IDESC = (2u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate), "r"(z));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar))
               : "memory");
}

struct Unit {
  int nt, mt, slot, poly;
};
// Unit u of k_bat_tc (n tile fastest, then m tile, poly, slot); tile counts are
// powers of two and the host keeps every unit index below 2^31.
__device__ __forceinline__ Unit decode(int u, int nt_shift, int mt_shift, int polys) {
  Unit r;
  r.nt = u & ((1 << nt_shift) - 1);
  u >>= nt_shift;
  r.mt = u & ((1 << mt_shift) - 1);
  u >>= mt_shift;
  r.slot = (unsigned)u / (unsigned)polys;
  r.poly = u - r.slot * polys;
  return r;
}

// Per-slot constants of the epilogue, reloaded only when the slot changes.
struct SlotCache {
  int slot = -1;
  ModC mc;
  VarC vc;                         // RED_MONTGOMERY / RED_BAT_LAZY constants of the slot
  const uint32_t* tab = nullptr;   // EPI_MUL table row of the slot
  uint32_t scal = 0;               // EPI_COMBINE / EPI_MODDOWN scalar of the slot
};

// Matrix dimensions of a launch: compile-time 256 for the 256 x 256 stages of
// N = 2^16 (DIM = 256), so every stride folds into an immediate, else the
// launch arguments (DIM = 0).
template <int DIM>
__device__ __forceinline__ int dim_rows(const Args& a) { return DIM ? DIM : a.rows_m; }
template <int DIM>
__device__ __forceinline__ int dim_nout(const Args& a) { return DIM ? DIM : a.nout; }
template <int DIM>
__device__ __forceinline__ int dim_kw(const Args& a) { return DIM ? DIM : a.kw; }

// Epilogue of one 128 x 256 accumulator tile, run by the 16 epilogue warps
// (TMEM lane quadrant warp % 4, column quarter (warp - 2) / 4): tcgen05.ld,
// byte recombination, Barrett, the fused position-wise op, stores.  Output
// position of (row m, output n): NMAJOR n*rows_m + m, else m*nout + n.  The
// operands of the fused op are read at the same positions before the
// accumulator is ready (16 consecutive words per thread when row major: four
// 16-byte loads).  Returns false when the wait for the accumulator gave up.
// RED (RedMode) selects the reductions: Barrett (RED_BARRETT_FAST: the exact
// 32-bit forms), or for the plain transforms of the variant plans Montgomery
// (every reduction) or BAT-lazy (the first reduction lazy, Barrett after).
template <int EPI, bool NMAJOR, int RED, int DIM>
__device__ __forceinline__ bool epilogue_tile(const Args& a, uint32_t tmem_acc, uint64_t* tfull, uint32_t parity,
                                              volatile int& abort, const Unit& w, bool store, int warp, int lane,
                                              SlotCache& sc) {
  static_assert(RED < RED_MONTGOMERY || EPI == EPI_NONE || EPI == EPI_MUL,
                "variant reductions only run the plain transform epilogues");
  constexpr bool FAST = RED == RED_BARRETT_FAST;
  constexpr int OUTS = 16;                     // outputs (64 columns) per thread and tile
  const int rows_m = dim_rows<DIM>(a), nout = dim_nout<DIM>(a);
  const int quad = warp & 3, part = (warp - 2) >> 2;
  constexpr int P0 = EPI == EPI_NONE ? 1 : OUTS;
  constexpr int P1 = EPI == EPI_MODDOWN ? OUTS : 1;
  if (w.slot != sc.slot) {
    sc.slot = w.slot;
    sc.mc = a.mods[a.limbs[w.slot]];
    if (RED >= RED_MONTGOMERY) sc.vc = a.varc[a.limbs[w.slot]];
    if (EPI == EPI_MUL) sc.tab = a.e.tab + (int64_t)a.e.trow[w.slot] * ((int64_t)rows_m * nout);
    if (EPI == EPI_COMBINE || EPI == EPI_MODDOWN) sc.scal = a.e.scal[w.slot];
  }
  const int m = w.mt * BM + quad * 32 + lane;
  const int n0 = w.nt * 64 + part * OUTS;
  const int64_t p0 = NMAJOR ? (int64_t)n0 * rows_m + m : (int64_t)m * nout + n0;
  uint32_t pre0[P0], pre1[P1];
  const uint32_t scal = sc.scal;
  bool add_base = false;
  if (EPI != EPI_NONE) {
    const uint32_t* src = EPI == EPI_MUL ? sc.tab + p0 : a.e.x.at(w.poly, w.slot) + p0;
    if (NMAJOR) {
#pragma unroll
      for (int j = 0; j < OUTS; ++j) pre0[j] = __ldg(src + (int64_t)j * rows_m);
    } else {
#pragma unroll
      for (int j = 0; j < OUTS / 4; ++j) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(src) + j);
        pre0[4 * j] = v.x;
        pre0[4 * j + 1] = v.y;
        pre0[4 * j + 2] = v.z;
        pre0[4 * j + 3] = v.w;
      }
    }
  }
  if (EPI == EPI_MODDOWN) {
    add_base = (a.e.base_mask >> ((unsigned)w.poly % (unsigned)a.e.base.E)) & 1u;
    if (add_base) {
      const uint4* b = reinterpret_cast<const uint4*>(a.e.base.at(w.poly, w.slot) + p0);
#pragma unroll
      for (int j = 0; j < OUTS / 4; ++j) {
        const uint4 v = __ldg(b + j);
        pre1[4 * j] = v.x;
        pre1[4 * j + 1] = v.y;
        pre1[4 * j + 2] = v.z;
        pre1[4 * j + 3] = v.w;
      }
    }
  }
  const ModC& mc = sc.mc;
  bool ok = mbar_wait(tfull, parity, abort, a.err, 4);
  ok = __all_sync(0xffffffffu, ok);
  if (!ok) return false;
  tc_fence_after();
  uint32_t* o = a.out + (int64_t)w.poly * a.out_ps + (int64_t)w.slot * a.out_ss + p0;
  const uint32_t q32 = (uint32_t)mc.q, m32 = (uint32_t)mc.m, sw = mc.s_w;
  // accumulator columns in quarters of 16 (four outputs): the next quarter's
  // tcgen05.ld is in flight while the current quarter is reduced
  const uint32_t tbase = tmem_acc + ((uint32_t)(quad * 32) << 16) + part * 64;
  uint32_t va[16], vb[16];
  tmem_ld16_issue(tbase, va);
  tmem_wait16(va);
#pragma unroll
  for (int chunk = 0; chunk < OUTS / 8; ++chunk) {
    uint32_t res[8];
    tmem_ld16_issue(tbase + chunk * 32 + 16, vb);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j == 4) {
        tmem_wait16(vb);
        if (chunk + 1 < OUTS / 8) tmem_ld16_issue(tbase + (chunk + 1) * 32, va);
      }
      const uint32_t* v = j < 4 ? va : vb;
      const int jv = j & 3;
      const int jj = chunk * 8 + j;
      const uint64_t z = combine4_mad(v[4 * jv], v[4 * jv + 1], v[4 * jv + 2], v[4 * jv + 3]);
      uint32_t r;
      if (RED == RED_MONTGOMERY)
        r = montgomery(z, q32, sc.vc.qinv);
      else if (RED == RED_BAT_LAZY && EPI == EPI_MUL)
        r = 0;   // the lazy value feeds the twiddle product below
      else
        r = FAST ? reduce_fast(z, q32, m32, sw) : barrett(z, mc);
      if (EPI == EPI_MUL) {
        if (RED == RED_MONTGOMERY)
          r = montgomery((uint64_t)r * pre0[jj], q32, sc.vc.qinv);
        else if (RED == RED_BAT_LAZY)
          r = barrett(bat_lazy(z, sc.vc.r) * pre0[jj], mc);
        else if (FAST)
          r = reduce_fast2(r * pre0[jj], __umulhi(r, pre0[jj]), q32, m32, sw);
        else
          r = barrett((uint64_t)r * pre0[jj], mc);
      } else if (EPI == EPI_COMBINE) {
        // x < 2^31 with beta < q and r < 2^32 keeps x beta + r below
        // 2^31 q + 2^32, where the fast form is exact; larger x take the 64-bit form
        const uint32_t x = pre0[jj];
        if (FAST && x < 0x80000000u) {
          const uint64_t zc = (uint64_t)x * scal + r;
          r = reduce_fast2((uint32_t)zc, (uint32_t)(zc >> 32), q32, m32, sw);
        } else {
          const uint64_t zc = (uint64_t)x * scal + r;
          r = FAST ? barrett_w32(zc, q32, m32, sw) : barrett(zc, mc);
        }
      } else if (EPI == EPI_MODDOWN) {
        // sub < 2^31 with P^-1 < q keeps the product below 2^31 q, where the
        // fast form is exact; larger operands take the 64-bit form
        const uint32_t x = pre0[jj];
        const uint32_t sub = x < r ? x + q32 - r : x - r;
        uint32_t t;
        if (FAST && sub < 0x80000000u)
          t = reduce_fast2(sub * scal, __umulhi(sub, scal), q32, m32, sw);
        else if (FAST)
          t = barrett_w32((uint64_t)sub * scal, q32, m32, sw);
        else
          t = barrett((uint64_t)sub * scal, mc);
        if (add_base) {
          const uint32_t s2 = pre1[jj] + t;
          r = s2 >= q32 ? s2 - q32 : s2;
        } else {
          r = t;
        }
      }
      res[j] = r;
    }
    if (store) {
      if (NMAJOR) {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[(int64_t)(chunk * 8 + j) * rows_m] = res[j];
      } else {
        // Lanes 2k and 2k+1 hold rows m and m+1 (1 KiB or more apart), eight
        // outputs each.  They swap halves so that each store instruction
        // writes whole 32-byte row segments: the first store row m
        // (even lane: its outputs 0-3, odd lane: the even lane's 4-7), the
        // second row m+1.
        const int odd = lane & 1;
        const uint4 lo = make_uint4(res[0], res[1], res[2], res[3]);
        const uint4 hi = make_uint4(res[4], res[5], res[6], res[7]);
        const uint4 x = odd ? lo : hi;
        uint4 y;
        y.x = __shfl_xor_sync(0xffffffffu, x.x, 1);
        y.y = __shfl_xor_sync(0xffffffffu, x.y, 1);
        y.z = __shfl_xor_sync(0xffffffffu, x.z, 1);
        y.w = __shfl_xor_sync(0xffffffffu, x.w, 1);
        uint32_t* base = o + chunk * 8 + odd * 4;
        *reinterpret_cast<uint4*>(base - (int64_t)odd * nout) = odd ? y : lo;
        *reinterpret_cast<uint4*>(base + (int64_t)(1 - odd) * nout) = odd ? hi : y;
      }
    }
    if (chunk + 1 < OUTS / 8) tmem_wait16(va);
  }
  return true;
}

template <int EPI, bool NMAJOR, int RED>
__global__ void __launch_bounds__(THREADS, 1) k_bat_tc(const __grid_constant__ CUtensorMap tmA,
                                                       const __grid_constant__ CUtensorMap tmB, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  Smem& S = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kst = a.kw / 32;
  const int mt_shift = __ffs(a.rows_m / BM) - 1, nt_shift = __ffs(a.nout / 64) - 1;
  const int units = a.slots * a.polys << (mt_shift + nt_shift);
  const int polys = (int)a.polys;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.tfull[i], 1);
      mbar_init(&S.tempty[i], 32 * EPI_WARPS);
    }
    mbar_init(&S.drain, 1);
    S.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmB) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(&S.tmem_base)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      uint32_t stage = 0, phase = 0;
      int issued = 0;
      for (int u = blockIdx.x; u < units && !S.abort; u += gridDim.x) {
        const Unit w = decode(u, nt_shift, mt_shift, polys);
        const int limb = a.limbs[w.slot];
        for (int ks = 0; ks < kst; ++ks) {
          if (!mbar_wait(&S.empty[stage], phase ^ 1, S.abort, a.err, 1)) break;
          mbar_expect_tx(&S.full[stage], A_STAGE + B_STAGE);
          tma_load_4d(S.a[stage], &tmA, &S.full[stage], ks * 32, w.mt * BM, w.slot, (int)w.poly);
          tma_load_2d(S.b[stage], &tmB, &S.full[stage], ks * BKB, limb * 4 * a.nout + w.nt * BN);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (S.abort) {
        // let the copies already issued land before the CTA exits
        for (int i = 0; i < STAGES && i < issued; ++i) {
          stage = stage == 0 ? STAGES - 1 : stage - 1;
          if (stage == STAGES - 1) phase ^= 1;
          const uint64_t t0 = globaltimer();
          while (!mbar_test(&S.full[stage], phase) && globaltimer() - t0 < WAIT_NS) __nanosleep(200);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      uint32_t stage = 0, phase = 0, acc = 0, aphase = 0;
      for (int u = blockIdx.x; u < units && !S.abort; u += gridDim.x) {
        if (!mbar_wait(&S.tempty[acc], aphase ^ 1, S.abort, a.err, 2)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        bool ok = true;
        for (int ks = 0; ks < kst; ++ks) {
          if (!mbar_wait(&S.full[stage], phase, S.abort, a.err, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t as = saddr(S.a[stage]), bs = saddr(S.b[stage]);
#pragma unroll
          for (int k = 0; k < BKB / 32; ++k)
            mma_i8(d, sw128_desc(as + 32 * k), sw128_desc(bs + 32 * k), (ks | k) != 0);
          mma_commit(&S.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&S.tfull[acc]);
        acc ^= 1;
        if (acc == 0) aphase ^= 1;
      }
      // every MMA issued by this thread has completed once `drain` flips
      mma_commit(&S.drain);
      const uint64_t t0 = globaltimer();
      while (!mbar_test(&S.drain, 0) && globaltimer() - t0 < WAIT_NS) __nanosleep(100);
    }
  } else {
    // ---------------- epilogue (warps 2..17) ----------------
    uint32_t acc = 0, aphase = 0;
    SlotCache sc;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const Unit w = decode(u, nt_shift, mt_shift, polys);
      if (!epilogue_tile<EPI, NMAJOR, RED, 0>(a, tmem + acc * BN, &S.tfull[acc], aphase, S.abort, w, true, warp,
                                               lane, sc))
        break;
      tc_fence_before();
      mbar_arrive(&S.tempty[acc]);
      acc ^= 1;
      if (acc == 0) aphase ^= 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
}

// ---------------------------------------------------------------------------
// Two-SM variant: a cluster of two CTAs issues tcgen05.mma.cta_group::2 with
// M = 256 (128 rows from each CTA's shared memory), N = 256.  Each CTA keeps
// its half of the B tile (128 rows x 4*kw bytes, kw <= 256) resident in shared
// memory for as long as the pair stays on one (limb, n tile) and streams only
// A, so a CTA reads 16 KiB from L2 per 512 tensor cycles instead of 48 KiB.
// Pairs form groups of n_tiles; the pairs of a group walk the same sequence of
// (slot, row-block pair) items, one n tile each, so the A tiles they share are
// read from L2 at about the same time.
//
// Roles per CTA as in k_bat_tc; only the leader (cluster rank 0) issues MMAs.
// Barriers: full[s] and bfull live in the leader and count the copies of both
// CTAs (TMA with .cta_group::2 signals the leader's barrier); empty[s],
// tfull[acc] and bempty live in both CTAs and are signalled by a multicast
// tcgen05.commit; tempty[acc] lives in the leader and counts one arrival per
// epilogue warp of both CTAs.  Every wait is bounded as in k_bat_tc; a
// cluster barrier keeps both CTAs alive until neither can signal the other.
constexpr int B2_ROWS = BN / 2;                  // B rows held per CTA
constexpr int B2_CHUNK = B2_ROWS * BKB;          // 16 KiB per 128-byte K chunk
constexpr int B2_CHUNKS = 8;                     // kw <= 256
constexpr int KPS = 2;                           // 128-byte K chunks per A stage (8 MMAs per stage)
constexpr int STAGES2 = 3;                       // A ring: 96 KiB in flight per CTA
constexpr uint32_t IDESC2 = (2u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)((2 * BM) >> 4) << 24);

struct Smem2 {
  uint8_t a[STAGES2][KPS * A_STAGE];
  uint8_t b[B2_CHUNKS][B2_CHUNK];
  uint64_t full[STAGES2];
  uint64_t empty[STAGES2];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t bfull, bempty, drain;
  uint32_t tmem_base;
  volatile int abort;
};
constexpr size_t SMEM2_BYTES = sizeof(Smem2) + 1024;
static_assert(SMEM2_BYTES <= 232448, "k_bat_tc2 shared memory exceeds 227 KiB");

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t mapa(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr(p)), "r"(rank));
  return r;
}
// Arrive on a barrier of either CTA of the cluster (the epilogue's release of
// an accumulator: tcgen05.fence::before_thread_sync orders its TMEM reads, no
// global memory ordering is needed, so the default CTA-scope release).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cl_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cl_addr) : "memory");
}
__device__ __forceinline__ void tma_load_4d_pair(void* dst, const CUtensorMap* tm, uint32_t bar_cl, int c0, int c1,
                                                 int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5, %6}], [%2];" ::"r"(saddr(dst)),
      "l"((uint64_t)tm), "r"(bar_cl), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* tm, uint32_t bar_cl, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(saddr(dst)),
      "l"((uint64_t)tm), "r"(bar_cl), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_l2_4d(const CUtensorMap* tm, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"((uint64_t)tm), "r"(c0),
               "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(IDESC2), "r"(accumulate), "r"(z));
}
// arrive on the barrier at this offset in both CTAs of the pair once the MMAs
// issued so far have completed
__device__ __forceinline__ void mma_commit_pair_both(uint64_t* bar) {
  const uint16_t mask = 3;
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                   saddr(bar)),
               "h"(mask)
               : "memory");
}
__device__ __forceinline__ void mma_commit_pair_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar))
               : "memory");
}

// Work of a pair: group g = pair / n_tiles over items [t0, t1) of the
// (slot, j) sequence (j = row-block pair, ipc per slot), n tile pair % n_tiles.
// The host keeps slots * ipc below 2^31.
struct PairWork {
  int t0, t1, ipc, rbs, nt, mt_shift;
};
template <int DIM>
__device__ __forceinline__ PairWork pair_work(const Args& a) {
  PairWork pw;
  const int n_tiles = dim_nout<DIM>(a) / 64;
  const int pair = blockIdx.x >> 1, groups = (gridDim.x >> 1) / n_tiles;
  const int g = pair / n_tiles;
  pw.nt = pair - g * n_tiles;
  pw.mt_shift = __ffs(dim_rows<DIM>(a) / BM) - 1;
  pw.rbs = (int)a.polys << pw.mt_shift;
  pw.ipc = (pw.rbs + 1) / 2;
  const int64_t total = (int64_t)a.slots * pw.ipc;
  pw.t0 = (int)(total * g / groups);
  pw.t1 = (int)(total * (g + 1) / groups);
  return pw;
}
// Walks the items of a pair in order without divisions.
struct PairIter {
  int slot, j;
  __device__ __forceinline__ PairIter(const PairWork& pw) : slot(pw.t0 / pw.ipc), j(pw.t0 - slot * pw.ipc) {}
  __device__ __forceinline__ void next(const PairWork& pw) {
    if (++j == pw.ipc) {
      j = 0;
      ++slot;
    }
  }
  // Row block of this CTA (the peer of an odd last pair repeats the leader's
  // row block and stores nothing).
  __device__ __forceinline__ Unit unit(const PairWork& pw, uint32_t rank, bool& valid) const {
    Unit w;
    w.slot = slot;
    int rb = 2 * j + (int)rank;
    valid = rb < pw.rbs;
    if (!valid) rb = 2 * j;
    w.poly = rb >> pw.mt_shift;
    w.mt = rb & ((1 << pw.mt_shift) - 1);
    w.nt = pw.nt;
    return w;
  }
};

template <int EPI, bool NMAJOR, int RED, int DIM>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    k_bat_tc2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  Smem2& S = *reinterpret_cast<Smem2*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int kst = dim_kw<DIM>(a) / 32;
  const PairWork pw = pair_work<DIM>(a);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES2; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.tfull[i], 1);
      mbar_init(&S.tempty[i], 2 * EPI_WARPS);
    }
    mbar_init(&S.bfull, 1);
    mbar_init(&S.bempty, 1);
    mbar_init(&S.drain, 1);
    S.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmB) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(&S.tmem_base)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      uint32_t stage = 0, phase = 0, bphase = 0;
      int prev_slot = -1;
      int issued = 0;
      PairIter it(pw);
      for (int t = pw.t0; t < pw.t1 && !S.abort; ++t, it.next(pw)) {
        bool valid;
        const Unit w = it.unit(pw, rank, valid);
        if (t + 1 < pw.t1) {
          // pull the next item's A rows into L2 while this item streams
          PairIter nx = it;
          nx.next(pw);
          bool nv;
          const Unit wn = nx.unit(pw, rank, nv);
          for (int kc = 0; kc < kst; ++kc) tma_prefetch_l2_4d(&tmA, kc * 32, wn.mt * BM, wn.slot, wn.poly);
        }
        if (w.slot != prev_slot) {
          // the MMAs that read the resident B half have completed
          if (!mbar_wait(&S.bempty, bphase ^ 1, S.abort, a.err, 11)) break;
          bphase ^= 1;
          const int limb = a.limbs[w.slot];
          if (rank == 0) mbar_expect_tx(&S.bfull, 2 * kst * B2_CHUNK);
          const uint32_t bar = mapa(&S.bfull, 0);
          for (int kc = 0; kc < kst; ++kc)
            tma_load_2d_pair(S.b[kc], &tmB, bar, kc * BKB, limb * 4 * dim_nout<DIM>(a) + w.nt * BN + (int)rank * B2_ROWS);
          prev_slot = w.slot;
        }
        for (int kc = 0; kc < kst; kc += KPS) {
          if (!mbar_wait(&S.empty[stage], phase ^ 1, S.abort, a.err, 12)) break;
          if (rank == 0) mbar_expect_tx(&S.full[stage], 2 * KPS * A_STAGE);
          const uint32_t bar = mapa(&S.full[stage], 0);
          for (int h = 0; h < KPS; ++h)
            tma_load_4d_pair(S.a[stage] + h * A_STAGE, &tmA, bar, (kc + h) * 32, w.mt * BM, w.slot, w.poly);
          ++issued;
          if (++stage == STAGES2) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (S.abort && rank == 0) {
        // let the copies already issued land before the CTA exits
        for (int i = 0; i < STAGES2 && i < issued; ++i) {
          stage = stage == 0 ? STAGES2 - 1 : stage - 1;
          if (stage == STAGES2 - 1) phase ^= 1;
          const uint64_t t0 = globaltimer();
          while (!mbar_test(&S.full[stage], phase) && globaltimer() - t0 < WAIT_NS) __nanosleep(200);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer (leader) ----------------
      uint32_t stage = 0, phase = 0, acc = 0, aphase = 0, bphase = 0;
      int prev_slot = -1;
      PairIter it(pw);
      for (int t = pw.t0; t < pw.t1 && !S.abort; ++t, it.next(pw)) {
        const int slot = it.slot;
        if (!mbar_wait(&S.tempty[acc], aphase ^ 1, S.abort, a.err, 13)) break;
        if (slot != prev_slot) {
          if (!mbar_wait(&S.bfull, bphase, S.abort, a.err, 14)) break;
          bphase ^= 1;
          prev_slot = slot;
        }
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        bool ok = true;
        for (int kc = 0; kc < kst; kc += KPS) {
          if (!mbar_wait(&S.full[stage], phase, S.abort, a.err, 15)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int h = 0; h < KPS; ++h) {
            const uint32_t as = saddr(S.a[stage] + h * A_STAGE), bs = saddr(S.b[kc + h]);
#pragma unroll
            for (int k = 0; k < BKB / 32; ++k)
              mma_i8_pair(d, sw128_desc(as + 32 * k), sw128_desc(bs + 32 * k), (kc | h | k) != 0);
          }
          mma_commit_pair_both(&S.empty[stage]);
          if (++stage == STAGES2) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_pair_both(&S.tfull[acc]);
        acc ^= 1;
        if (acc == 0) aphase ^= 1;
        if (t + 1 == pw.t1 || it.j + 1 == pw.ipc) mma_commit_pair_both(&S.bempty);
      }
      // every MMA issued by this thread has completed once `drain` flips
      mma_commit_pair_local(&S.drain);
      const uint64_t t0 = globaltimer();
      while (!mbar_test(&S.drain, 0) && globaltimer() - t0 < WAIT_NS) __nanosleep(100);
    }
  } else {
    // ---------------- epilogue (both CTAs, warps 2..17) ----------------
    uint32_t acc = 0, aphase = 0;
    SlotCache sc;
    PairIter it(pw);
    for (int t = pw.t0; t < pw.t1; ++t, it.next(pw)) {
      bool valid;
      const Unit w = it.unit(pw, rank, valid);
      if (!epilogue_tile<EPI, NMAJOR, RED, DIM>(a, tmem + acc * BN, &S.tfull[acc], aphase, S.abort, w, valid, warp,
                                                 lane, sc))
        break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa(&S.tempty[acc], 0));
      acc ^= 1;
      if (acc == 0) aphase ^= 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
}

// Strided batched transpose of limb-polynomials: out[lp][c][r] = in[lp][r][c].
__global__ void k_transpose_lp(LP in, uint32_t* __restrict__ out, int64_t lps, int slots, int R, int C) {
  __shared__ uint32_t tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  const int64_t N = (int64_t)R * C;
  for (int64_t lp = blockIdx.z; lp < lps; lp += gridDim.z) {
    const uint32_t* src = in.p + (lp / slots) * in.ps + (lp % slots) * in.ss;
    uint32_t* dst = out + lp * N;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) tile[i][threadIdx.x] = src[(int64_t)(r0 + i) * C + c0 + threadIdx.x];
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) dst[(int64_t)(c0 + i) * R + r0 + threadIdx.x] = tile[threadIdx.x][i];
    __syncthreads();
  }
}

// The driver's tensor-map encoder (one entry point for all devices).
std::atomic<PFN_cuTensorMapEncodeTiled_v12000> g_encode{nullptr};

int init_driver() {
  if (!g_encode.load(std::memory_order_acquire)) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    CROSS_CHECK_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !fn) {
      set_error("cuTensorMapEncodeTiled is not available from the driver");
      return CROSS_ERR_UNSUPPORTED;
    }
    g_encode.store((PFN_cuTensorMapEncodeTiled_v12000)fn, std::memory_order_release);
  }
  return CROSS_OK;
}

int encode(CUtensorMap* tm, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
           const cuuint64_t* strides, const cuuint32_t* box) {
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = g_encode.load(std::memory_order_acquire)(tm, dt, rank, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return CROSS_ERR_CUDA;
  }
  return CROSS_OK;
}

// Tensor map of A: (kw words, rows, slots, polys) with word strides.
int make_tmap_a(CUtensorMap* tm, const uint32_t* base, int kw, int rows, int slots, int64_t polys, int64_t ss,
                int64_t ps) {
  const int64_t mat = (int64_t)kw * rows;
  if (slots == 1 || ss == 0) ss = mat;
  if (polys == 1 || ps == 0) ps = ss * slots;
  if (((uintptr_t)base & 15) || (ss * 4) % 16 || (ps * 4) % 16) {
    set_error("tcgen05 NTT: limb-polynomial base and strides must be 16-byte aligned");
    return CROSS_ERR_UNSUPPORTED;
  }
  cuuint64_t dims[4] = {(cuuint64_t)kw, (cuuint64_t)rows, (cuuint64_t)slots, (cuuint64_t)polys};
  cuuint64_t strides[3] = {(cuuint64_t)kw * 4, (cuuint64_t)ss * 4, (cuuint64_t)ps * 4};
  cuuint32_t box[4] = {32, (cuuint32_t)BM, 1, 1};
  return encode(tm, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, base, dims, strides, box);
}

// Tensor map of a plan's B matrices: (4*kw bytes, M*4*nout rows), boxes of
// `rows` rows (BN for k_bat_tc, BN / 2 for one CTA of k_bat_tc2).
int make_tmap_b(CUtensorMap* tm, const uint8_t* base, int kw, int nout, int M, int rows) {
  cuuint64_t dims[2] = {(cuuint64_t)4 * kw, (cuuint64_t)M * 4 * nout};
  cuuint64_t strides[1] = {(cuuint64_t)4 * kw};
  cuuint32_t box[2] = {(cuuint32_t)BKB, (cuuint32_t)rows};
  return encode(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides, box);
}

template <int EPI, bool NM, int RED>
int launch(const CUtensorMap& tmA, const CUtensorMap& tmB, const Args& a, cudaStream_t st) {
  CROSS_CHECK_CUDA(cudaFuncSetAttribute(k_bat_tc<EPI, NM, RED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)SMEM_BYTES));
  const int64_t units = (int64_t)a.slots * a.polys * (a.rows_m / BM) * (a.nout / 64);
  const int sms = device_sm_count();
  const unsigned grid = (unsigned)(units < sms ? units : sms);
  k_bat_tc<EPI, NM, RED><<<grid, THREADS, SMEM_BYTES, st>>>(tmA, tmB, a);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

template <int EPI, bool NM, int RED, int DIM>
int launch2(const CUtensorMap& tmA, const CUtensorMap& tmB, const Args& a, cudaStream_t st) {
  auto kern = k_bat_tc2<EPI, NM, RED, DIM>;
  CROSS_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM2_BYTES));
  // clusters of two 225 KiB CTAs that fit at once (compile-time cluster dims);
  // every instantiation has the same resources
  static PerDevice pairs_cache;
  const int max_pairs = pairs_cache.get([&] {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(device_sm_count() & ~1));
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = SMEM2_BYTES;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (const void*)kern, &cfg) != cudaSuccess || n < 1) {
      (void)cudaGetLastError();
      n = device_sm_count() / 2;
    }
    return n;
  });
  const int m_tiles = a.rows_m / BM, n_tiles = a.nout / 64;
  const int64_t rbs = a.polys * m_tiles, total = (int64_t)a.slots * ((rbs + 1) / 2);
  if (total == 0) return CROSS_OK;
  int64_t groups = max_pairs / n_tiles;
  if (groups < 1) groups = 1;
  if (groups > total) groups = total;
  kern<<<(unsigned)(2 * groups * n_tiles), THREADS, SMEM2_BYTES, st>>>(tmA, tmB, a);
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  return CROSS_OK;
}

// One contraction stage over polys x slots limb-polynomials.  tmB2 is the
// half-height map of the same B matrices (used by k_bat_tc2 when kw <= 256).
int stage(const cross_ntt_plan_s* P, const CUtensorMap& tmB, const CUtensorMap& tmB2, bool nmajor, const Epi& e,
          const uint32_t* A,
          int64_t a_ps, int64_t a_ss, int rows_m, int kw, int nout, LPo out, int64_t polys, int slots,
          const uint16_t* limbs, cudaStream_t st) {
  CUtensorMap tmA;
  int rc = make_tmap_a(&tmA, A, kw, rows_m, slots, polys, a_ss, a_ps);
  if (rc) return rc;
  // unit and item indices are 32-bit inside the kernels
  if ((int64_t)slots * polys * (rows_m / BM) * (nout / 64) >= ((int64_t)1 << 31)) {
    set_error("tcgen05 stage: %lld limb-polynomials exceed one launch", (long long)(polys * slots));
    return CROSS_ERR_UNSUPPORTED;
  }
  Args a{out.p, out.ps, out.ss, limbs, slots, polys, rows_m, kw, nout, P->mods, P->varc, P->tc_err, e};
  // row-major outputs are written with 16-byte stores
  if (!nmajor && (((uintptr_t)out.p & 15) || (slots > 1 && out.ss % 4) || (polys > 1 && out.ps % 4))) {
    set_error("tcgen05 stage: the output base and strides must be 16-byte aligned");
    return CROSS_ERR_INVALID_ARG;
  }
  if (!nmajor && e.op != EPI_NONE) {
    // row-major operands are read with 16-byte loads
    const View& x = e.op == EPI_MUL ? View{e.tab, 0, 0, 0, 1} : e.x;
    bool al = ((uintptr_t)x.p & 15) == 0 && x.ps % 4 == 0 && x.es % 4 == 0 && x.ss % 4 == 0;
    if (e.op == EPI_MUL) al = al && ((int64_t)rows_m * nout) % 4 == 0;
    if (e.op == EPI_MODDOWN && e.base_mask)
      al = al && ((uintptr_t)e.base.p & 15) == 0 && e.base.ps % 4 == 0 && e.base.es % 4 == 0 && e.base.ss % 4 == 0;
    if (!al) {
      set_error("tcgen05 stage: epilogue operands must be 16-byte aligned");
      return CROSS_ERR_UNSUPPORTED;
    }
  }
  const bool f = P->tc_fast != 0;
  const bool pair = P->tc_pair && kw <= 32 * B2_CHUNKS && kw % (32 * KPS) == 0;
  const bool d256 = rows_m == 256 && nout == 256 && kw == 256;
  if (P->red == CROSS_REDUCTION_MONTGOMERY || P->red == CROSS_REDUCTION_BAT_LAZY) {
    // variant plans: the plain transform stages (ntt_exec_tc's three epilogue
    // shapes) with run-time dimensions
#define CROSS_TC_VAR(OP, NM)                                                                       \
  return P->red == CROSS_REDUCTION_MONTGOMERY                                                     \
             ? (pair ? launch2<OP, NM, RED_MONTGOMERY, 0>(tmA, tmB2, a, st)                       \
                     : launch<OP, NM, RED_MONTGOMERY>(tmA, tmB, a, st))                           \
             : (pair ? launch2<OP, NM, RED_BAT_LAZY, 0>(tmA, tmB2, a, st)                         \
                     : launch<OP, NM, RED_BAT_LAZY>(tmA, tmB, a, st))
    if (e.op == EPI_MUL && nmajor) CROSS_TC_VAR(EPI_MUL, true);
    if (e.op == EPI_NONE && nmajor) CROSS_TC_VAR(EPI_NONE, true);
    if (e.op == EPI_NONE && !nmajor) CROSS_TC_VAR(EPI_NONE, false);
#undef CROSS_TC_VAR
    set_error("tcgen05 stage: epilogue %d (output major %d) not available with reduction %d", e.op, (int)nmajor,
              P->red);
    return CROSS_ERR_UNSUPPORTED;
  }
#define CROSS_TC_LAUNCH(OP, NM)                                                                                  \
  return pair ? (d256 ? (f ? launch2<OP, NM, RED_BARRETT_FAST, 256>(tmA, tmB2, a, st)                             \
                           : launch2<OP, NM, RED_BARRETT, 256>(tmA, tmB2, a, st))                                 \
                      : (f ? launch2<OP, NM, RED_BARRETT_FAST, 0>(tmA, tmB2, a, st)                               \
                           : launch2<OP, NM, RED_BARRETT, 0>(tmA, tmB2, a, st)))                                  \
              : (f ? launch<OP, NM, RED_BARRETT_FAST>(tmA, tmB, a, st) : launch<OP, NM, RED_BARRETT>(tmA, tmB, a, st))
  switch (e.op) {
    case EPI_NONE:
      if (nmajor) CROSS_TC_LAUNCH(EPI_NONE, true);
      CROSS_TC_LAUNCH(EPI_NONE, false);
    case EPI_MUL:
      if (nmajor) CROSS_TC_LAUNCH(EPI_MUL, true);
      CROSS_TC_LAUNCH(EPI_MUL, false);
    case EPI_COMBINE:
      if (nmajor) break;
      CROSS_TC_LAUNCH(EPI_COMBINE, false);
    case EPI_MODDOWN:
      if (nmajor) break;
      CROSS_TC_LAUNCH(EPI_MODDOWN, false);
  }
#undef CROSS_TC_LAUNCH
  set_error("tcgen05 stage: unsupported epilogue %d (output major %d)", e.op, (int)nmajor);
  return CROSS_ERR_UNSUPPORTED;
}


// ---------------------------------------------------------------------------
// N = 2^12 (64 x 64): both contraction stages of a transform in one launch.
// A CTA takes one limb-polynomial at a time and keeps everything in shared
// memory: the two stages' B matrices (256 rows x 256 B each, TMA,
// SWIZZLE_128B), the stage-1 A tile (written by the threads in the same
// swizzled K-major layout: transposed for the forward transform, which
// contracts over r, as is for the inverse, which contracts over c) and the
// stage-2 A tile, which the stage-1 epilogue writes directly (byte
// recombination, Barrett, twiddle multiply, Barrett).  The polynomial's 64
// rows fill both halves of each 128-row A tile, so the accumulator's lanes
// 64..127 repeat lanes 0..63 and the warps of the upper lane quadrants reduce
// the other half of the outputs: eight outputs per thread and stage.  Per
// stage 8 tcgen05.mma kind::i8 of M = 128, N = 256, K = 32 into one 256-column
// TMEM accumulator; the stage-2 epilogue (recombination, Barrett) stores the
// natural-order result.  Bounded waits as in k_bat_tc (codes 41 to 44).
constexpr int T64_THREADS = 512;   // 16 warps: four per TMEM lane quadrant, 8 outputs each per stage
struct Smem64 {
  uint8_t b1[2][256 * 128];    // stage-1 B: two 128-byte K chunks of 256 rows
  uint8_t b2[2][256 * 128];    // stage-2 B
  uint8_t a1[2][128 * 128];    // stage-1 A: two K chunks of 128 rows
  uint8_t a2[2][128 * 128];    // stage-2 A
  uint64_t bbar, mbar, drain;
  uint32_t tmem_base;
  volatile int abort;
};
constexpr size_t SMEM64_BYTES = sizeof(Smem64) + 1024;
static_assert(SMEM64_BYTES <= 232448, "k_ntt64 shared memory exceeds 227 KiB");

struct Args64 {
  LP in;
  LPo out;
  int64_t polys;
  int slots;
  const uint16_t* limbs;
  const ModC* mods;
  const uint32_t* tw;   // forward: tf_step2 [limb][z][c]; inverse: intt_tf_step2 transposed [limb][l][r]
  int* err;
};

// byte offset of (row, 16-byte chunk k16 of the 256-byte K extent) in a
// 128-row, two-chunk SWIZZLE_128B K-major tile
__device__ __forceinline__ uint32_t sw_off(int row, int k16) {
  return (uint32_t)((k16 >> 3) * (128 * 128) + (row >> 3) * 1024 + (row & 7) * 128 + (((k16 & 7) ^ (row & 7)) << 4));
}

// Issue the 8 MMAs of one stage (A: 128 rows x 256 B, B: 256 rows x 256 B) and commit.
__device__ __forceinline__ void ntt64_mma(uint32_t tmem, const uint8_t* a, const uint8_t* b, uint64_t* bar) {
#pragma unroll
  for (int kc = 0; kc < 2; ++kc)
#pragma unroll
    for (int k = 0; k < 4; ++k)
      mma_i8(tmem, sw128_desc(saddr(a + kc * 128 * 128) + 32 * k), sw128_desc(saddr(b + kc * 256 * 128) + 32 * k),
             (kc | k) != 0);
  mma_commit(bar);
}

template <bool INV, bool FAST>
__global__ void __launch_bounds__(T64_THREADS, 1)
    k_ntt64(const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ CUtensorMap tmB2, const Args64 a) {
  extern __shared__ uint8_t smem_raw[];
  Smem64& S = *reinterpret_cast<Smem64*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int64_t total = (int64_t)a.slots * a.polys;   // one limb-polynomial per item
  const int64_t i0 = total * blockIdx.x / gridDim.x, i1 = total * (blockIdx.x + 1) / gridDim.x;
  if (t == 0) {
    mbar_init(&S.bbar, 1);
    mbar_init(&S.mbar, 1);
    mbar_init(&S.drain, 1);
    S.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmB1) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmB2) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(&S.tmem_base)),
                 "r"(256)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;
  uint32_t bphase = 0, mphase = 0;
  int cur_slot = -1;
  // epilogue role: the A tiles hold the polynomial's 64 rows twice (rows
  // 0..63 and 64..127), so TMEM lanes 64..127 repeat lanes 0..63.  Lane
  // quadrant q = warp % 4 gives row mm (quadrants 0-1 and 2-3 cover the 64 rows
  // each) and the output half (quadrants 0-1: outputs 0..31, 2-3: 32..63); the
  // output eighth h = warp / 4 within the half gives the thread's eight
  // outputs ob .. ob + 7, accumulator columns 4 ob .. 4 ob + 31
  const int q = warp & 3, h = warp >> 2;
  const int mm = (32 * q + lane) & 63, ob = 32 * (q >> 1) + 8 * h;
  for (int64_t it = i0; it < i1; ++it) {
    const int slot = (int)(it / a.polys);
    const int64_t p = it - (int64_t)slot * a.polys;
    const int limb = a.limbs[slot];
    if (slot != cur_slot && t == 0) {
      // the MMAs that read the previous slot's B tiles have completed (waited below)
      mbar_expect_tx(&S.bbar, 4 * 256 * 128);
      for (int kc = 0; kc < 2; ++kc) {
        tma_load_2d(S.b1[kc], &tmB1, &S.bbar, kc * 128, limb * 256);
        tma_load_2d(S.b2[kc], &tmB2, &S.bbar, kc * 128, limb * 256);
      }
    }
    // stage-1 A tile from global memory, each row stored twice
    {
      const uint32_t* x = a.in.p + p * a.in.ps + (int64_t)slot * a.in.ss;
      if (!INV) {
        // forward: A rows c, K words r (the transpose of X[r][c])
        const int c = t & 63, rg = t >> 6;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int r0 = 32 * i + 4 * rg;
          uint4 v;
          v.x = __ldg(x + (r0 + 0) * 64 + c);
          v.y = __ldg(x + (r0 + 1) * 64 + c);
          v.z = __ldg(x + (r0 + 2) * 64 + c);
          v.w = __ldg(x + (r0 + 3) * 64 + c);
          *reinterpret_cast<uint4*>(&S.a1[0][0] + sw_off(c, r0 >> 2)) = v;
          *reinterpret_cast<uint4*>(&S.a1[0][0] + sw_off(64 + c, r0 >> 2)) = v;
        }
      } else {
        // inverse: A rows r, K words c (X as stored)
        const int c4 = t & 15;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int r = (t >> 4) + 32 * i;
          const uint4 v = __ldg(reinterpret_cast<const uint4*>(x + r * 64) + c4);
          *reinterpret_cast<uint4*>(&S.a1[0][0] + sw_off(r, c4)) = v;
          *reinterpret_cast<uint4*>(&S.a1[0][0] + sw_off(64 + r, c4)) = v;
        }
      }
    }
    // stage-1 twiddles of this thread's outputs, in flight during the MMA
    const ModC mc = a.mods[limb];
    const uint32_t q32 = (uint32_t)mc.q, m32 = (uint32_t)mc.m, sw = mc.s_w;
    uint32_t tw[8];
    {
      const uint32_t* tb = a.tw + (int64_t)limb * 4096 + mm;
#pragma unroll
      for (int o = 0; o < 8; ++o) tw[o] = __ldg(tb + (ob + o) * 64);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (t == 0) {
      bool ok = true;
      if (slot != cur_slot) {
        ok = mbar_wait(&S.bbar, bphase, S.abort, a.err, 41);
        bphase ^= 1;
      }
      if (ok) {
        tc_fence_after();
        ntt64_mma(tmem, &S.a1[0][0], &S.b1[0][0], &S.mbar);
        if (!mbar_wait(&S.mbar, mphase, S.abort, a.err, 42)) S.abort = 1;
      } else {
        S.abort = 1;
      }
    }
    cur_slot = slot;
    mphase ^= 1;
    __syncthreads();
    if (S.abort) break;
    tc_fence_after();
    // stage-1 epilogue: Y = Barrett(Barrett(sum) x twiddle) into the stage-2 A
    // tile (row: output index o, stored twice; K word: this thread's row mm)
    {
      uint32_t v[32];
      tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + 4 * ob, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int o = ob + j;
        const uint64_t z = combine4_mad(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        const uint32_t wv = tw[j];
        uint32_t r;
        if (FAST) {
          r = reduce_fast(z, q32, m32, sw);
          r = reduce_fast2(r * wv, __umulhi(r, wv), q32, m32, sw);
        } else {
          r = barrett(z, mc);
          r = barrett((uint64_t)r * wv, mc);
        }
        *reinterpret_cast<uint32_t*>(&S.a2[0][0] + sw_off(o, mm >> 2) + 4 * (mm & 3)) = r;
        *reinterpret_cast<uint32_t*>(&S.a2[0][0] + sw_off(64 + o, mm >> 2) + 4 * (mm & 3)) = r;
      }
    }
    tc_fence_before();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (t == 0) {
      tc_fence_after();
      ntt64_mma(tmem, &S.a2[0][0], &S.b2[0][0], &S.mbar);
      if (!mbar_wait(&S.mbar, mphase, S.abort, a.err, 43)) S.abort = 1;
    }
    mphase ^= 1;
    __syncthreads();
    if (S.abort) break;
    tc_fence_after();
    // stage-2 epilogue: Barrett, natural-order stores of this polynomial
    {
      uint32_t* y = a.out.p + p * a.out.ps + (int64_t)slot * a.out.ss;
      uint32_t v[32];
      tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + 4 * ob, v);
      uint32_t res[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint64_t z = combine4_mad(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        res[j] = FAST ? reduce_fast(z, q32, m32, sw) : barrett(z, mc);
      }
      if (!INV) {
        // forward: Z[z][n], this thread's row z = mm, outputs n = ob .. ob + 7
        uint4* d = reinterpret_cast<uint4*>(y + mm * 64 + ob);
        d[0] = make_uint4(res[0], res[1], res[2], res[3]);
        d[1] = make_uint4(res[4], res[5], res[6], res[7]);
      } else {
        // inverse: Z[l][c], this thread's column c = mm, rows l = ob .. ob + 7
#pragma unroll
        for (int j = 0; j < 8; ++j) y[(ob + j) * 64 + mm] = res[j];
      }
    }
    tc_fence_before();
    __syncthreads();
  }
  if (t == 0 && S.abort) {
    // let anything still in flight land before TMEM is freed and the CTA exits
    mma_commit(&S.drain);
    const uint64_t t0 = globaltimer();
    while (!mbar_test(&S.drain, 0) && globaltimer() - t0 < WAIT_NS) __nanosleep(100);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");
}

}  // namespace tc

bool tc_supported(int r, int c) {
  auto ok = [](int x) { return x >= 128 && x <= 1024 && (x & (x - 1)) == 0; };
  return ok(r) && ok(c);
}

// B matrices of the tensor-core path from the reference BAT arrays:
//   bat (X, 4 q, Y, 4 p, M); `x_is_out` when the first axis indexes the output n
//   (ntt step 1 / intt step 3: n = z or l, w = r), else the second spatial axis does
//   (ntt step 3 / intt step 1: w = c, n = n or l).
//   dst[m][n][p][w][q] bytes: the four q-bytes of one (m, n, p, w) are one
//   little-endian word, written in order per limb.
void pack_tc(const uint8_t* bat, int X, int Y, int M, bool x_is_out, std::vector<uint8_t>& dst) {
  const int nout = x_is_out ? X : Y, kw = x_is_out ? Y : X;
  dst.resize((size_t)M * 4 * nout * 4 * kw);
  const size_t lw = (size_t)4 * nout * kw;     // words per limb
  const size_t qs = (size_t)Y * 4 * M;         // source stride of q
  for (int n = 0; n < nout; ++n)
    for (int p = 0; p < 4; ++p)
      for (int w = 0; w < kw; ++w) {
        const int x = x_is_out ? n : w, y = x_is_out ? w : n;
        const uint8_t* s = bat + (((size_t)x * 4 * Y + y) * 4 + p) * M;
        uint8_t* d = dst.data() + (((size_t)n * 4 + p) * kw + w) * 4;
        for (int m = 0; m < M; ++m) {
          const uint32_t word = (uint32_t)s[m] | (uint32_t)s[qs + m] << 8 | (uint32_t)s[2 * qs + m] << 16 |
                                (uint32_t)s[3 * qs + m] << 24;
          std::memcpy(d + m * lw * 4, &word, 4);
        }
      }
}

int tc_plan_init(cross_ntt_plan_s* P, const uint8_t* ntt1, const uint8_t* ntt3, const uint8_t* intt1,
                 const uint8_t* intt3, const uint32_t* intt_tw) {
  // 64 x 64 Barrett plans (N = 2^12) get the single-launch kernel k_ntt64 for
  // their plain transforms (the B matrices and maps below serve both kernels)
  const bool n64 = P->r == 64 && P->c == 64 && P->red == CROSS_REDUCTION_BARRETT;
  if (!tc_supported(P->r, P->c) && !n64) return CROSS_OK;
  int rc = tc::init_driver();
  if (rc) return rc;
  const int R = P->r, C = P->c, M = P->M;
  std::vector<uint8_t> buf;
  pack_tc(ntt1, R, R, M, true, buf);
  if ((rc = upload_vec(&P->tc_col_fwd, buf))) return rc;
  pack_tc(intt3, R, R, M, true, buf);
  if ((rc = upload_vec(&P->tc_col_inv, buf))) return rc;
  pack_tc(ntt3, C, C, M, false, buf);
  if ((rc = upload_vec(&P->tc_row_fwd, buf))) return rc;
  pack_tc(intt1, C, C, M, false, buf);
  if ((rc = upload_vec(&P->tc_row_inv, buf))) return rc;
  // intt twiddle as [limb][l][r] (output index major) for the row-stage epilogue
  std::vector<uint32_t> tw((size_t)M * R * C);
  for (int l = 0; l < C; ++l)
    for (int r = 0; r < R; ++r) {
      const uint32_t* s = intt_tw + ((size_t)r * C + l) * M;
      for (int m = 0; m < M; ++m) tw[((size_t)m * C + l) * R + r] = s[m];
    }
  if ((rc = upload_vec(&P->tc_tw_inv, tw))) return rc;
  std::vector<int> zero(1, 0);
  if ((rc = upload(&P->tc_err, zero.data(), 1))) return rc;
  for (int h = 0; h < 2; ++h) {
    const int rows = h ? tc::BN / 2 : tc::BN;
    if ((rc = tc::make_tmap_b(h ? &P->tm2_col_fwd : &P->tm_col_fwd, P->tc_col_fwd, R, R, M, rows))) return rc;
    if ((rc = tc::make_tmap_b(h ? &P->tm2_col_inv : &P->tm_col_inv, P->tc_col_inv, R, R, M, rows))) return rc;
    if ((rc = tc::make_tmap_b(h ? &P->tm2_row_fwd : &P->tm_row_fwd, P->tc_row_fwd, C, C, M, rows))) return rc;
    if ((rc = tc::make_tmap_b(h ? &P->tm2_row_inv : &P->tm_row_inv, P->tc_row_inv, C, C, M, rows))) return rc;
  }
  // two-SM kernel unless CROSS_B200_TC_1SM=1 (kept for comparison runs)
  const char* one = getenv("CROSS_B200_TC_1SM");
  P->tc_pair = !(one && one[0] == '1');
  // FAST selects reduce_fast in every epilogue and barrett_w32 in the combine /
  // ModDown epilogues.
  bool fast = true;
  for (const ModC& mc : P->mods_host) fast = fast && reduce_fast_ok(mc);
  P->tc_fast = fast ? 1 : 0;
  P->tc = !n64;
  P->tc64 = n64;
  return CROSS_OK;
}

void tc_plan_free(cross_ntt_plan_s* P) {
  dfree(P->tc_col_fwd);
  dfree(P->tc_col_inv);
  dfree(P->tc_row_fwd);
  dfree(P->tc_row_inv);
  dfree(P->tc_tw_inv);
  dfree(P->tc_err);
}

// NTT / INTT on the tensor cores.  tmp holds 2 * polys * slots * N words.
//   ntt:  [transpose natural input] -> column stage (x T2, output index major)
//         -> row stage (row major) with epi
//   intt: row stage (x iT2, output index major) -> column stage with epi,
//         output index major (natural coefficients) or row major (transposed)
int ntt_exec_tc(const cross_ntt_plan_s* P, bool inverse, LP in, int in_layout, LPo out, int out_layout,
                int64_t polys, int slots, const uint16_t* limbs, const Epi& epi, uint32_t* tmp, cudaStream_t st) {
  const int R = P->r, C = P->c;
  const int64_t N = (int64_t)R * C, lps = polys * slots;
  uint32_t* t1 = tmp;
  uint32_t* t2 = tmp + lps * N;
  Epi tw;
  tw.op = EPI_MUL;
  tw.trow = limbs;
  int rc;
  if (!inverse) {
    const uint32_t* A = in.p;
    int64_t aps = in.ps, ass = in.ss;
    if (in_layout == COEF_NATURAL) {
      dim3 blk(32, 8), grd(C / 32, R / 32, (unsigned)(lps < 65535 ? lps : 65535));
      tc::k_transpose_lp<<<grd, blk, 0, st>>>(in, t1, lps, slots, R, C);
      count_launch();
      CROSS_CHECK_CUDA(cudaGetLastError());
      A = t1;
      aps = slots * N;
      ass = N;
    }
    // column stage: A = X^T (C rows x R words), out Y[z][c] = out[n][m], x T2[z][c]
    tw.tab = P->tw_fwd;
    if ((rc = tc::stage(P, P->tm_col_fwd, P->tm2_col_fwd, true, tw, A, aps, ass, C, R, R, LPo{t2, slots * N, N}, polys, slots, limbs,
                        st)))
      return rc;
    // row stage: A = Y (R rows x C words), out Z[z][n] = out[m][n]
    return tc::stage(P, P->tm_row_fwd, P->tm2_row_fwd, false, epi, t2, slots * N, N, R, C, C, out, polys, slots, limbs, st);
  }
  // row stage: A = X (R rows x C words), out Y^T[l][r] = out[n][m], x iT2[r][l]
  tw.tab = P->tc_tw_inv;
  if ((rc = tc::stage(P, P->tm_row_inv, P->tm2_row_inv, true, tw, in.p, in.ps, in.ss, R, C, C, LPo{t1, slots * N, N}, polys, slots,
                      limbs, st)))
    return rc;
  // column stage: A = Y^T (C rows x R words), out Z[l'][c'] = out[n][m] (natural)
  // or Z^T[c'][l'] = out[m][n] (transposed)
  return tc::stage(P, P->tm_col_inv, P->tm2_col_inv, out_layout == COEF_NATURAL, epi, t1, slots * N, N, C, R, R, out, polys, slots,
                   limbs, st);
}

// NTT / INTT of polys x slots limb-polynomials of a 64 x 64 plan, natural
// coefficient order on both sides, in one launch.
int ntt64_run(const cross_ntt_plan_s* P, bool inverse, LP in, LPo out, int64_t polys, int slots,
              const uint16_t* limbs, cudaStream_t st) {
  const int64_t total = (int64_t)slots * polys;
  if (total == 0) return CROSS_OK;
  tc::Args64 a{in, out, polys, slots, limbs, P->mods, inverse ? P->tc_tw_inv : P->tw_fwd, P->tc_err};
  const int sms = device_sm_count();
  const unsigned grid = (unsigned)(total < sms ? total : sms);
  const CUtensorMap& b1 = inverse ? P->tm_row_inv : P->tm_col_fwd;
  const CUtensorMap& b2 = inverse ? P->tm_col_inv : P->tm_row_fwd;
  auto go = [&](auto kern) -> int {
    CROSS_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc::SMEM64_BYTES));
    kern<<<grid, tc::T64_THREADS, tc::SMEM64_BYTES, st>>>(b1, b2, a);
    count_launch();
    CROSS_CHECK_CUDA(cudaGetLastError());
    return CROSS_OK;
  };
  if (P->tc_fast) return inverse ? go(tc::k_ntt64<true, true>) : go(tc::k_ntt64<false, true>);
  return inverse ? go(tc::k_ntt64<true, false>) : go(tc::k_ntt64<false, false>);
}

}  // namespace cross

// ---------------------------------------------------------------------------
// Throughput probe of tcgen05.mma kind::i8: the peak that the contraction
// kernels' roofline fractions are quoted against.  Every CTA keeps one A tile
// (128 rows x 128 B) and one B tile (N rows x 128 B), SWIZZLE_128B, filled
// with hashed bytes so the data is not all zero, in shared memory; one thread
// issues kchunks x 4 back-to-back MMAs of K = 32 into a 256-column TMEM
// accumulator -- M = 128, N = 256 per CTA (pair = 0) or M = 256, N = 256 per
// cluster of two CTAs with cta_group::2 (pair = 1, the form of k_bat_tc2) --
// and commits once.  No global memory is read; the only wait is the bounded
// wait for that commit (code 31 in *err on expiry).
namespace cross {
namespace tc {

constexpr int PROBE_THREADS = 128;
// more than half an SM's shared memory, so that no SM holds two probe CTAs
// (only the first 48 KiB + barrier are used)
constexpr size_t PROBE_SMEM = 160 * 1024;

template <bool PAIR>
__global__ void __launch_bounds__(PROBE_THREADS, 1) k_i8_probe(int64_t kchunks, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // A: 128 rows x 128 B; B: N rows x 128 B (256 rows for one CTA, 128 per CTA
  // of a pair), so the barrier follows 48 KiB of operands
  uint8_t* As = base;
  uint8_t* Bs = base + A_STAGE;
  uint64_t* bar = reinterpret_cast<uint64_t*>(base + A_STAGE + B_STAGE);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  volatile int& abort = *reinterpret_cast<volatile int*>(tslot + 1);
  const int warp = threadIdx.x >> 5;
  const uint32_t rank = PAIR ? cluster_rank() : 0;
  for (int i = threadIdx.x; i < (A_STAGE + B_STAGE) / 4; i += PROBE_THREADS) {
    uint32_t h = (uint32_t)i * 2654435761u ^ (blockIdx.x * 0x9E3779B9u);
    h ^= h >> 15;
    h *= 2246822519u;
    h ^= h >> 13;
    reinterpret_cast<uint32_t*>(base)[i] = h;
  }
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    if (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tslot)), "r"(256)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tslot)), "r"(256)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
  }
  // the generic-proxy fill must be visible to the tensor cores' async proxy
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  if (threadIdx.x == 0 && rank == 0) {
    const uint32_t as = saddr(As), bs = saddr(Bs);
    for (int64_t i = 0; i < kchunks; ++i) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (PAIR)
          mma_i8_pair(tmem, sw128_desc(as + 32 * k), sw128_desc(bs + 32 * k), (i | k) != 0);
        else
          mma_i8(tmem, sw128_desc(as + 32 * k), sw128_desc(bs + 32 * k), (i | k) != 0);
      }
    }
    if (PAIR)
      mma_commit_pair_both(bar);
    else
      mma_commit(bar);
  }
  if (threadIdx.x == 0) mbar_wait(bar, 0, abort, err, 31);
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();
  tc_fence_after();
  if (warp == 1) {
    if (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");
  }
}

template <bool PAIR>
int launch_probe(int64_t kchunks, int* err, int* ctas, cudaStream_t st) {
  auto kern = k_i8_probe<PAIR>;
  CROSS_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PROBE_SMEM));
  const int sms = device_sm_count();
  int grid = sms;
  if (PAIR) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)(sms & ~1));
    cfg.blockDim = dim3(PROBE_THREADS);
    cfg.dynamicSmemBytes = PROBE_SMEM;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (const void*)kern, &cfg) != cudaSuccess || n < 1) {
      (void)cudaGetLastError();
      n = sms / 2;
    }
    // one CTA per SM (the shared-memory request keeps a second one out)
    grid = 2 * (n < sms / 2 ? n : sms / 2);
    cfg.gridDim = dim3((unsigned)grid);
    CROSS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, kchunks, err));
  } else {
    kern<<<grid, PROBE_THREADS, PROBE_SMEM, st>>>(kchunks, err);
  }
  count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  *ctas = grid;
  return CROSS_OK;
}

}  // namespace tc
}  // namespace cross

// Self-test of the bounded waits every tensor-core kernel uses: one warp waits
// on an mbarrier that nothing arrives on, through the same bounded wait, and
// must give up after bound_ns, record code 51 in the error word and return.
namespace cross {
namespace tc {
__device__ int g_wait_selftest_err;

__global__ void k_wait_selftest(uint64_t bound_ns) {
  __shared__ uint64_t bar;
  __shared__ volatile int abort;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // phase 0 never completes: no thread arrives on bar
  const bool ok = mbar_wait_for(&bar, 0, abort, &g_wait_selftest_err, 51, bound_ns);
  if (__any_sync(0xffffffffu, ok) && threadIdx.x == 0) atomicExch(&g_wait_selftest_err, 52);
}
}  // namespace tc
}  // namespace cross

extern "C" int cross_wait_selftest(uint64_t bound_ns, void* stream) {
  CROSS_REQUIRE(bound_ns >= 1000 && bound_ns <= 1000000000ull,
                "cross_wait_selftest: bound_ns=%llu outside 1 us .. 1 s", (unsigned long long)bound_ns);
  int e = 0;
  CROSS_CHECK_CUDA(cudaMemcpyToSymbolAsync(cross::tc::g_wait_selftest_err, &e, sizeof(int), 0,
                                           cudaMemcpyHostToDevice, (cudaStream_t)stream));
  cross::tc::k_wait_selftest<<<1, 32, 0, (cudaStream_t)stream>>>(bound_ns);
  cross::count_launch();
  CROSS_CHECK_CUDA(cudaGetLastError());
  CROSS_CHECK_CUDA(cudaMemcpyFromSymbolAsync(&e, cross::tc::g_wait_selftest_err, sizeof(int), 0,
                                             cudaMemcpyDeviceToHost, (cudaStream_t)stream));
  CROSS_CHECK_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  if (e == 51) {
    cross::set_error("bounded wait expired after %llu ns as intended (code %d)", (unsigned long long)bound_ns, e);
    return CROSS_ERR_TIMEOUT;
  }
  cross::set_error("cross_wait_selftest: the wait on a barrier nothing arrives on ended with code %d", e);
  return CROSS_ERR_CUDA;
}

extern "C" int cross_tc_i8_probe(int pair, int64_t kchunks, int* err, int* ctas, void* stream) {
  CROSS_REQUIRE(err && ctas && kchunks >= 1 && kchunks <= (1 << 20),
                "cross_tc_i8_probe: need err, ctas and 1 <= kchunks <= 2^20");
  return pair ? cross::tc::launch_probe<true>(kchunks, err, ctas, (cudaStream_t)stream)
              : cross::tc::launch_probe<false>(kchunks, err, ctas, (cudaStream_t)stream);
}
