// GEMM on the B200 tensor cores (tcgen05 / TMEM / TMA), sm_100a.
//
// C[b] = epilogue(alpha * A[b] · B[b]) for the math-plus Backend.matmul / Backend.linear path
// (packages/tensor-cpu/src/index.ts:755-774; the reference computes it with gemmNT,
// packages/tensor-core/src/kernels.ts:299-362, in f64 on the host).
//
// One persistent CTA per SM, 10 warps, warp-specialised:
//   warp 0      TMA producer: A / B tiles into a STAGES-deep shared-memory ring (mbarrier full/empty)
//   warp 1      MMA issuer: one thread issues tcgen05.mma into a TMEM accumulator and commits
//               stage releases and accumulator completion to mbarriers; also owns the TMEM allocation
//   warps 2..9  epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes 32*(w%4)..+31; two
//               warps per lane quadrant split the columns), apply alpha / +bias / exact-erf GELU,
//               convert, stage 32-row x 128-byte swizzled blocks in shared memory and TMA-store
//               them (bounds clipped by the tensor map)
// Two TMEM accumulators let the epilogue of tile i overlap the main loop of tile i+1. The linear
// (B K-major) kernel on CTA pairs gives each epilogue warp two staging blocks (5 stages instead of 6
// to make room), so a block is staged while the store of the one before it still reads: with
// K = 768 (GPT-2's projections) the epilogue is no longer hidden, and out-proj + residual took
// 58.5 us against 64.1, fc + GELU 176.5 against 180.6 (the matmul kernel of the batched
// configuration keeps 6 stages and one block: it measured slower the other way).
//
// Operand layouts, all with the 128-byte swizzle:
//   A        K-major (row-major [M,K]); box {BK, 128}
//   B [N,K]  K-major (the linear weight);  box {BK, BN}
//   B [K,N]  MN-major (the matmul operand); BN/64 boxes {64, BK}, one per 128-byte N chunk
// f16 / bf16 inputs use kind::f16 (BK = 64, MMA K = 16, BN = 256, 4 stages).
// f32 inputs use 3xTF32 (kind::tf32, BK = 32, MMA K = 8, BN = 128, 3 stages): a prologue splits each
// operand into tf32 hi + lo parts (K-major), and the main loop accumulates lo·hi + hi·lo + hi·hi.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "gelu.cuh"
#include "mpc_internal.h"
#include "sm100.cuh"

namespace mpc {
namespace gemm {

enum Kind { kHalf = 0, kTF32x3 = 1 };

struct Params {
  int M, N, K;
  int tiles_m, tiles_n, tiles_total;
  int k_blocks;
  int group_m;
  int brank;
  int bshape[4];
  int a_bstride[4];  // batch strides in whole matrices (0 = broadcast)
  int b_bstride[4];
  float alpha;
  const float *bias;
  int epilogue;
  int out_dtype;
  uint32_t idesc;  // tcgen05 instruction descriptor (operand format, B major, M, N)
  int *err;
  unsigned long long timeout_ns;
  int ndst;            // output maps in use (1 unless the product is stored to several matrices)
  const void *resid;   // MPC_EPI_RESIDUAL: [batch, M, N] in the output type, added last
  int resid_vec;       // resid rows start 16-byte aligned (vector loads)
  void *c_direct;      // non-null: C [batch, M, N] whose rows are not 16-byte aligned, written with
                       // plain stores from the staged block instead of TMA
  int splits;          // 3xTF32: K halves per output tile (1 or 2); with 2 the halves add into a zeroed C
  int kb_split;        // K blocks per half
};

// Work unit u of the persistent loop: its output tile and K-block range. Only the 3xTF32 kernel splits
// K (two halves of one tile on different SMs, reduce-added into C); everything else has one unit per tile.
template <int KIND>
__device__ __forceinline__ void unit_range(const Params &p, int u, int &tile, int &kb0, int &kb1, bool &first) {
  if constexpr (KIND == kTF32x3) {
    const int sp = u % p.splits;
    tile = u / p.splits;
    kb0 = sp * p.kb_split;
    kb1 = min(kb0 + p.kb_split, p.k_blocks);
    first = sp == 0;
  } else {
    tile = u;
    kb0 = 0;
    kb1 = p.k_blocks;
    first = true;
  }
}

// The operand maps and NDST output maps; each 32 x 32 output block is stored through c[0..ndst).
template <int NDST>
struct MapsT {
  CUtensorMap a, b, a_lo, b_lo, c[NDST];
};
using Maps = MapsT<1>;
constexpr int kMaxDst = 8;

template <int KIND, bool B_MN, int BN, int STAGES, bool PAIR = false, int EPI_BUFS = 1>
struct Cfg {
  static constexpr int BM = 128;                   // rows of A / C per CTA
  static constexpr int TILE_M = PAIR ? 256 : 128;  // rows of one output tile (a CTA pair shares one)
  static constexpr int BNL = PAIR ? BN / 2 : BN;   // rows of B held by one CTA
  static constexpr int ES = KIND == kHalf ? 2 : 4;  // operand element bytes
  static constexpr int BK = 128 / ES;               // elements in one 128-byte row
  static constexpr int UK = KIND == kHalf ? 16 : 8;  // K of one tcgen05.mma
  static constexpr int KSTEPS = BK / UK;
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BNL * 128;
  static constexpr int NOPS = KIND == kHalf ? 1 : 2;
  static constexpr int STAGE_BYTES = NOPS * (A_BYTES + B_BYTES);
  static constexpr int EPI_WARPS = 8;
  static constexpr int THREADS = 32 * (2 + EPI_WARPS);
  static constexpr int EPI_BYTES = EPI_WARPS * 4096 * EPI_BUFS;  // EPI_BUFS 32-row x 128-byte staging blocks per warp
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES;
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation must be a power of two");
  static_assert(!(KIND == kTF32x3 && B_MN), "3xTF32 operands are always K-major");
  static_assert(!(PAIR && KIND != kHalf), "CTA pairs run the f16 / bf16 kernel only");
};

__device__ __forceinline__ void tile_coords(const Params &p, int tile, int &b, int &mt, int &nt) {
  const int per_batch = p.tiles_m * p.tiles_n;
  b = tile / per_batch;
  const int r = tile - b * per_batch;
  const int group = p.group_m * p.tiles_n;
  const int g = r / group;
  const int first_m = g * p.group_m;
  const int gm = min(p.tiles_m - first_m, p.group_m);
  const int rg = r - g * group;
  mt = first_m + rg % gm;
  nt = rg / gm;
}

__device__ __forceinline__ void batch_index(const Params &p, int b, int &ia, int &ib) {
  ia = 0;
  ib = 0;
#pragma unroll
  for (int d = 3; d >= 0; --d) {  // static indices keep the parameter arrays out of local memory
    if (d < p.brank) {
      const int i = b % p.bshape[d];
      b /= p.bshape[d];
      ia += i * p.a_bstride[d];
      ib += i * p.b_bstride[d];
    }
  }
}


// alpha, +bias and GELU on one 32-column chunk of this warp's 32 rows (lane = row). The math is
// written once; only the packing below depends on the output type.
template <bool GELU_OK = true>
__device__ __forceinline__ void epilogue_math(const Params &p, float (&f)[32], int col0, int lane,
                                              bool add_bias = true) {
  if (p.alpha != 1.0f) {
#pragma unroll
    for (int j = 0; j < 32; ++j) f[j] *= p.alpha;
  }
  if ((p.epilogue & MPC_EPI_BIAS) && add_bias) {
    // Every lane adds the same 32 bias values: uniform 16-byte loads (one broadcast each) when the
    // chunk is whole and aligned, else one load per lane and shuffles.
    if (col0 + 32 <= p.N && !(reinterpret_cast<uintptr_t>(p.bias + col0) & 15)) {
      const float4 *b4 = reinterpret_cast<const float4 *>(p.bias + col0);
#pragma unroll
      for (int j = 0; j < 8; ++j) {  // paired f32 adds
        using namespace gelu_detail;
        const float4 bv = __ldg(b4 + j);
        const float2 s0 = unpk(add2(pk(f[4 * j], f[4 * j + 1]), pk(bv.x, bv.y)));
        const float2 s1 = unpk(add2(pk(f[4 * j + 2], f[4 * j + 3]), pk(bv.z, bv.w)));
        f[4 * j] = s0.x, f[4 * j + 1] = s0.y, f[4 * j + 2] = s1.x, f[4 * j + 3] = s1.y;
      }
    } else {
      const int c = col0 + lane;
      const float bl = c < p.N ? __ldg(p.bias + c) : 0.0f;
#pragma unroll
      for (int j = 0; j < 32; ++j) f[j] += __shfl_sync(0xffffffffu, bl, j);
    }
  }
  if (GELU_OK && (p.epilogue & MPC_EPI_GELU)) {
#pragma unroll
    for (int j = 0; j < 32; j += 2) gelu_erf_f32x2(f[j], f[j + 1]);
  }
}

// The 16-bit residual R[b, row, col0 .. col0+31] as four 16-byte loads (rows below M, whole aligned
// chunks; zeros otherwise).
__device__ __forceinline__ void load_resid16(const Params &p, int b, int row, int col0, uint4 (&v)[4]) {
  if (row < p.M && col0 + 32 <= p.N) {
    const uint4 *r = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(p.resid) +
                                                     (((int64_t)b * p.M + row) * p.N + col0));
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = r[j];
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = make_uint4(0, 0, 0, 0);
  }
}

__device__ __forceinline__ void add_resid16(float (&f)[32], const uint4 (&v)[4], bool bf) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t lo = w[e] & 0xFFFFu, hi = w[e] >> 16;
      f[8 * j + 2 * e] += bf ? __uint_as_float(lo << 16) : __half2float(__ushort_as_half((unsigned short)lo));
      f[8 * j + 2 * e + 1] += bf ? __uint_as_float(hi << 16) : __half2float(__ushort_as_half((unsigned short)hi));
    }
  }
}

// + R[b, row, col0 .. col0+31] (the residual, in the output type) for the lane's row.
__device__ __forceinline__ void add_residual(const Params &p, float (&f)[32], int b, int row, int col0) {
  if (row >= p.M) return;
  const int64_t base = ((int64_t)b * p.M + row) * p.N + col0;
  const int ncol = p.N - col0;
  if (p.out_dtype == MPC_F32) {
    const float *r = static_cast<const float *>(p.resid) + base;
    if (ncol >= 32 && p.resid_vec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 v = reinterpret_cast<const float4 *>(r)[j];
        f[4 * j] += v.x, f[4 * j + 1] += v.y, f[4 * j + 2] += v.z, f[4 * j + 3] += v.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncol) f[j] += r[j];
    }
    return;
  }
  const uint16_t *r = static_cast<const uint16_t *>(p.resid) + base;
  const bool bf = p.out_dtype == MPC_BF16;
  auto widen = [bf](uint32_t h) {
    return bf ? __uint_as_float(h << 16) : __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
  };
  if (ncol >= 32 && p.resid_vec) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 v = reinterpret_cast<const uint4 *>(r)[j];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        f[8 * j + 2 * e] += widen(w[e] & 0xFFFFu);
        f[8 * j + 2 * e + 1] += widen(w[e] >> 16);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < ncol) f[j] += widen(r[j]);
  }
}

// Writes row `lane` of a 32-row x 128-byte staging block in the 128-byte swizzle the store map
// expects (16-byte chunk j of a row at chunk j ^ (row & 7); bank-conflict free). An f32 chunk of
// 32 columns fills the row; a 16-bit chunk fills half of it (`half` selects which), so 16-bit
// outputs go out as 32 x 64-column stores.
__device__ __forceinline__ void stage_row(uint8_t *buf, const float (&f)[32], int out_dtype, int lane, int half) {
  uint8_t *row = buf + lane * 128;
  if (out_dtype == MPC_F32) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<uint4 *>(row + ((j ^ (lane & 7)) << 4)) =
          make_uint4(__float_as_uint(f[4 * j]), __float_as_uint(f[4 * j + 1]), __float_as_uint(f[4 * j + 2]),
                     __float_as_uint(f[4 * j + 3]));
  } else {
    uint32_t w[16];
    if (out_dtype == MPC_BF16) {
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        __nv_bfloat162 h2 = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
        w[e] = *reinterpret_cast<uint32_t *>(&h2);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        __half2 h2 = __floats2half2_rn(f[2 * e], f[2 * e + 1]);
        w[e] = *reinterpret_cast<uint32_t *>(&h2);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint4 *>(row + (((4 * half + j) ^ (lane & 7)) << 4)) =
          make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
  }
}

// PAIR: a cluster of two CTAs computes one 256 x BN tile with M = 256 tensor-core instructions
// issued by the even CTA. Each CTA loads its 128 rows of A and half of B's BN rows (counting the
// bytes on the even CTA's `full` barrier), holds its 128 rows of the accumulator in its own tensor
// memory and runs its own epilogue; the even CTA's MMA commits release both CTAs' slots and
// accumulators, and both CTAs' epilogue warps release the accumulator on the even CTA.
// RES16: the epilogue adds a 16-bit residual (no GELU), loading each chunk's residual while the chunk
// before it is stored; a separate instantiation so that the other epilogues keep their registers.
template <int KIND, bool B_MN, int BN, int STAGES, int NDST, bool PAIR, bool RES16 = false, int EPI_BUFS = 1>
__global__ void __launch_bounds__(320, 1) gemm_kernel(const __grid_constant__ MapsT<NDST> maps, const Params p) {
  using C = Cfg<KIND, B_MN, BN, STAGES, PAIR, EPI_BUFS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *stages = smem;
  uint8_t *epi = smem + STAGES * C::STAGE_BYTES;
  uint64_t *full = reinterpret_cast<uint64_t *>(epi + C::EPI_BYTES);
  uint64_t *empty = full + STAGES;
  uint64_t *acc_full = empty + STAGES;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *drain = acc_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0;  // 0: the CTA that issues the MMAs
  const int first_tile = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int tile_step = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], C::EPI_WARPS * (PAIR ? 2 : 1));
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&maps.a);
    tma_prefetch_desc(&maps.b);
    tma_prefetch_desc(&maps.c[0]);
    if constexpr (KIND == kTF32x3) {
      tma_prefetch_desc(&maps.a_lo);
      tma_prefetch_desc(&maps.b_lo);
    }
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();  // both CTAs' barriers are initialised before either signals the other's
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // 3xTF32 launches overlap their set-up with the split prologue (programmatic dependent launch):
  // the hi / lo planes and C's zeros are read only after the prologue has completed.
  if constexpr (KIND == kTF32x3) grid_dependency_wait();
  // Cluster addresses: the even CTA's `full` and `acc_empty` barriers (where both CTAs count),
  // and the odd CTA's `empty` and `acc_full` barriers (which the even CTA's commits release).
  const uint32_t full_lead = PAIR ? cluster_addr(full, 0) : 0;
  const uint32_t acc_empty_lead = PAIR ? cluster_addr(acc_empty, 0) : 0;
  const uint32_t empty_odd = PAIR ? cluster_addr(empty, 1) : 0;
  const uint32_t acc_full_odd = PAIR ? cluster_addr(acc_full, 1) : 0;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int u = first_tile; ok && u < p.tiles_total; u += tile_step) {
        int tile, kb0, kb1, b, mt, nt, ia, ib;
        bool first;
        unit_range<KIND>(p, u, tile, kb0, kb1, first);
        tile_coords(p, tile, b, mt, nt);
        batch_index(p, b, ia, ib);
        const int m_base = mt * C::TILE_M + static_cast<int>(rank) * C::BM;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.err, kErrWaitProducer, p.timeout_ns)) {
            ok = false;
            break;
          }
          uint8_t *sa = stages + stage * C::STAGE_BYTES;
          uint8_t *sb = sa + C::A_BYTES;
          if constexpr (PAIR) {
            // Both CTAs' bytes complete the even CTA's barrier, which the even CTA arms.
            if (rank == 0) mbar_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
            const uint32_t bar = full_lead + stage * 8;
            const int n_base = nt * BN + static_cast<int>(rank) * C::BNL;
            tma_load_3d_pair(&maps.a, bar, sa, kb * C::BK, m_base, ia);
            if constexpr (B_MN) {
#pragma unroll
              for (int j = 0; j < C::BNL / 64; ++j)
                tma_load_3d_pair(&maps.b, bar, sb + j * (C::BK * 128), n_base + j * 64, kb * C::BK, ib);
            } else {
              tma_load_3d_pair(&maps.b, bar, sb, kb * C::BK, n_base, ib);
            }
            ++issued;
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
            continue;
          }
          mbar_expect_tx(&full[stage], C::STAGE_BYTES);
          tma_load_3d(&maps.a, &full[stage], sa, kb * C::BK, m_base, ia);
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_3d(&maps.b, &full[stage], sb + j * (C::BK * 128), nt * BN + j * 64, kb * C::BK, ib);
          } else {
            tma_load_3d(&maps.b, &full[stage], sb, kb * C::BK, nt * BN, ib);
          }
          if constexpr (KIND == kTF32x3) {
            uint8_t *sa2 = sb + C::B_BYTES;
            uint8_t *sb2 = sa2 + C::A_BYTES;
            tma_load_3d(&maps.a_lo, &full[stage], sa2, kb * C::BK, m_base, ia);
            tma_load_3d(&maps.b_lo, &full[stage], sb2, kb * C::BK, nt * BN, ib);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok && !(PAIR && rank == 1)) {
        // Let the copies already in flight land before shared memory goes away: wait on the
        // full barriers of the (up to STAGES) most recently armed slots. (The odd CTA of a pair
        // counts its bytes on the even CTA's barriers; it gave up only after a full timeout
        // without a released slot, long after its last copies landed.)
        const int n = issued < STAGES ? issued : STAGES;
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < n; ++i) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1;
          }
          volatile int never = 0;
          mbar_wait(&full[s], ph, &never, p.err, kErrWaitProducer, p.timeout_ns);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (one thread; the even CTA's for a pair) ----------------
    if (lane == 0 && rank == 0) {
      const uint32_t idesc_rt = p.idesc;
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int u = first_tile; ok && u < p.tiles_total; u += tile_step, ++local) {
        int tile, kb0, kb1;
        bool first;
        unit_range<KIND>(p, u, tile, kb0, kb1, first);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag, p.err, kErrWaitAccEmpty, p.timeout_ns)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err, kErrWaitConsumer, p.timeout_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stages + stage * C::STAGE_BYTES);
          const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
          for (int ks = 0; ks < C::KSTEPS; ++ks) {
            const uint64_t ad = make_sdesc(a_addr + ks * (C::UK * C::ES), 16, 1024);
            const uint64_t bd = B_MN ? make_sdesc(b_addr + ks * (C::UK * 128), C::BK * 128, 1024)
                                     : make_sdesc(b_addr + ks * (C::UK * C::ES), 16, 1024);
            const uint32_t accum = (kb != kb0 || ks) ? 1u : 0u;
            if constexpr (PAIR) {
              mma_f16_ss_pair(d_tmem, ad, bd, idesc_rt, accum);
            } else if constexpr (KIND == kHalf) {
              mma_f16_ss(d_tmem, ad, bd, idesc_rt, accum);
            } else {
              const uint32_t a2 = b_addr + C::B_BYTES;
              const uint32_t b2 = a2 + C::A_BYTES;
              const uint64_t ad2 = make_sdesc(a2 + ks * (C::UK * C::ES), 16, 1024);
              const uint64_t bd2 = make_sdesc(b2 + ks * (C::UK * C::ES), 16, 1024);
              mma_tf32_ss(d_tmem, ad2, bd, idesc_rt, accum);  // lo · hi
              mma_tf32_ss(d_tmem, ad, bd2, idesc_rt, 1u);     // hi · lo
              mma_tf32_ss(d_tmem, ad, bd, idesc_rt, 1u);      // hi · hi
            }
          }
          if constexpr (PAIR) {  // the slot is free in both CTAs once these MMAs have read it
            tc_commit_pair(smem_u32(&empty[stage]));
            tc_commit_pair(empty_odd + stage * 8);
          } else {
            tc_commit(&empty[stage]);  // the slot is free once these MMAs have read it
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if constexpr (PAIR) {
          tc_commit_pair(smem_u32(&acc_full[acc]));
          tc_commit_pair(acc_full_odd + acc * 8);
        } else {
          tc_commit(&acc_full[acc]);
        }
      }
      // Every MMA this thread issued has completed once `drain` flips.
      if constexpr (PAIR)
        tc_commit_pair(smem_u32(drain));
      else
        tc_commit(drain);
      volatile int never = 0;
      mbar_wait(drain, 0, &never, p.err, kErrWaitConsumer, p.timeout_ns);
    }
  } else {
    // ---------------- epilogue (warps 2..9) ----------------
    const int ew = warp - 2;
    const int q = warp & 3;  // TMEM lane quadrant this warp may access (hardware rule: warp % 4)
    constexpr int COLS = BN / 2;  // each of the two warps of a quadrant takes half the columns
    const int col_base = (ew >> 2) * COLS;
    uint8_t *const buf0 = epi + ew * 4096 * EPI_BUFS;
    uint8_t *buf = buf0;
    int nblk = 0;  // staging blocks this warp has filled (the next one is nblk % EPI_BUFS)
    int local = 0;
    for (int u = first_tile; u < p.tiles_total; u += tile_step, ++local) {
      int tile, kb0, kb1, b, mt, nt;
      bool first;
      unit_range<KIND>(p, u, tile, kb0, kb1, first);
      tile_coords(p, tile, b, mt, nt);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_warp(&acc_full[acc], acc_phase, abort_flag, p.err, kErrWaitAccFull, p.timeout_ns)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN + col_base;
      const int row0 = mt * C::TILE_M + static_cast<int>(rank) * C::BM + q * 32;
      // The chunk loop; PRE (the RES16 kernel) has each chunk's 16-bit residual loaded while the chunk
      // before it is staged and stored.
      auto chunks = [&](auto pre) {
        constexpr bool PRE = decltype(pre)::value;
        uint32_t r[32];
        uint4 rv[4];
        const int colt = nt * BN + col_base;
        tmem_ld32(t_row, r);
        if constexpr (PRE) load_resid16(p, b, row0 + lane, colt, rv);
#pragma unroll 1
        for (int c = 0; c < COLS / 32; ++c) {
          tmem_ld_wait(r);
          float f[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]);
          if (c + 1 < COLS / 32) {
            tmem_ld32(t_row + (c + 1) * 32, r);  // next chunk's load overlaps this chunk's math
          } else {
            // This warp's share of the accumulator is in registers: release it to the MMA warp.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              if constexpr (PAIR)
                mbar_arrive_cluster(acc_empty_lead + acc * 8);
              else
                mbar_arrive(&acc_empty[acc]);
            }
          }
          const int col0 = nt * BN + col_base + c * 32;
          if constexpr (PRE) {
            epilogue_math<false>(p, f, col0, lane);
            if (col0 + 32 <= p.N)
              add_resid16(f, rv, p.out_dtype == MPC_BF16);
            else
              add_residual(p, f, b, row0 + lane, col0);
            // the next chunk's residual is in flight while this chunk is staged and stored
            if (c + 1 < COLS / 32) load_resid16(p, b, row0 + lane, colt + (c + 1) * 32, rv);
          } else {
            epilogue_math(p, f, col0, lane, first);  // a second K half adds no bias
            if (p.epilogue & MPC_EPI_RESIDUAL) add_residual(p, f, b, row0 + lane, col0);
          }
          // f32: one 32 x 32 store per chunk; 16-bit: chunks pair up into one 32 x 64 store
          const bool wide = p.out_dtype != MPC_F32;
          const int half = wide ? (c & 1) : 0;
          if (half == 0) {
            buf = buf0 + (nblk % EPI_BUFS) * 4096;
            ++nblk;
            if (lane == 0) tma_store_wait_read<EPI_BUFS - 1>();  // the store that last read this block is done
            __syncwarp();
          }
          stage_row(buf, f, p.out_dtype, lane, half);
          if ((!wide || half == 1) && p.c_direct) {
            // Row by row from the staged block: the warp writes one row's 32 (f32) or 64 (16-bit)
            // consecutive outputs per step, undoing the 128-byte swizzle.
            __syncwarp();
            const int cs = col0 - 32 * half;
            // The row pointer steps by N per row and the column bounds are fixed for the block; eight
            // rows per unrolled step (the GPT-2 LM head: 2.93 ms with four rows per step and per-row
            // index arithmetic, 2.44 ms like this; unrolling all 32 rows gained 2% more but made the
            // kernel spill). Half-word pairs measured faster than shifted 4-byte stores for rows
            // starting 2 bytes past a 4-byte boundary (3.96 ms), and than one 4-byte store per lane
            // on the rows that start 4-byte aligned with half-word pairs on the others (2.52 ms).
            const size_t rb0 = ((size_t)b * p.M + row0) * (size_t)p.N + cs;
            const int rows = p.M - row0 < 32 ? p.M - row0 : 32;
            if (!wide) {
              float *rp = static_cast<float *>(p.c_direct) + rb0;
              const bool colok = cs + lane < p.N;
#pragma unroll 8
              for (int rr = 0; rr < 32; ++rr, rp += p.N) {
                const uint32_t v = *reinterpret_cast<const uint32_t *>(buf + rr * 128 + (((lane >> 2) ^ (rr & 7)) << 4) +
                                                                       ((lane & 3) << 2));
                if (rr < rows && colok) rp[lane] = __uint_as_float(v);
              }
            } else {
              uint16_t *rp = static_cast<uint16_t *>(p.c_direct) + rb0;
              const int c0 = cs + 2 * lane;
              const bool ok0 = c0 < p.N, ok1 = c0 + 1 < p.N;
#pragma unroll 8
              for (int rr = 0; rr < 32; ++rr, rp += p.N) {
                const uint32_t v = *reinterpret_cast<const uint32_t *>(buf + rr * 128 + (((lane >> 2) ^ (rr & 7)) << 4) +
                                                                       ((lane & 3) << 2));
                if (rr < rows) {
                  if (ok0) rp[2 * lane] = static_cast<uint16_t>(v & 0xffffu);
                  if (ok1) rp[2 * lane + 1] = static_cast<uint16_t>(v >> 16);
                }
              }
            }
            __syncwarp();  // the block may be staged again
          } else if (!wide || half == 1) {
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              const int cs = col0 - 32 * half;
              if (row0 < p.M && cs < p.N) {
                if constexpr (KIND == kTF32x3) {
                  if (p.splits > 1)  // the two K halves add into C (zeroed before the launch)
                    tma_reduce_add_3d(&maps.c[0], buf, cs, row0, b);
                  else
                    tma_store_3d(&maps.c[0], buf, cs, row0, b);
                } else if constexpr (NDST == 1) {
                  tma_store_3d(&maps.c[0], buf, cs, row0, b);
                } else {  // the first destination rotates with the tile and warp: spread the peers' load
                  const int first = (tile + ew) % p.ndst;
                  for (int d = 0; d < p.ndst; ++d) {
                    const int t = first + d < p.ndst ? first + d : first + d - p.ndst;
                    tma_store_3d(&maps.c[t], buf, cs, row0, b);
                  }
                }
              }
              tma_store_commit();
            }
          }
        }
      };
      if constexpr (RES16)
        chunks(std::true_type{});
      else
        chunks(std::false_type{});
    }
    if (lane == 0) {
      tma_store_wait_all<0>();
      if constexpr (NDST > 1) {  // blocks stored to other GPUs are visible system-wide at kernel end
        asm volatile("fence.proxy.async.global;" ::: "memory");
        __threadfence_system();
      }
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncwarp();
  if constexpr (PAIR)
    cluster_sync();  // neither CTA frees tensor memory or leaves while the other may signal it
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---- 3xTF32 prologue: x = hi + lo with hi, lo tf32 values (round to nearest) ----------------
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// The 3xTF32 prologue, one launch: A's rows split into hi / lo planes, B's rows split (B [N,K]) or
// B [K,N] split and transposed to [N,K], and C zeroed when split-K halves add into it. The grid is
// cut into consecutive block ranges, one per part. It lets the GEMM launch at once (the GEMM waits
// for the prologue's completion before it reads the planes).
struct SplitJob {
  const float *a;
  float *a_hi, *a_lo;
  int64_t a_rows;
  const float *b;
  float *b_hi, *b_lo;
  int64_t b_rows;  // rows of B [N,K] (b_trans 0)
  int b_trans, nb, n;  // b_trans 1: B [nb][K][N] transposed to [nb][N][ld]
  int64_t k, ld;       // operand K and the planes' K pitch
  float *c;            // zeroed when non-null
  int64_t c_floats;
  unsigned ax, ay;      // A part: ax x ay blocks
  unsigned bx, by, bz;  // B part: bx x by (x bz) blocks
  unsigned cblocks;     // C part
};

// Row-major [rows, cols] -> [rows, ld] hi / lo (columns cols..ld-1 zero) by the gx x gy blocks of
// one part: rows walk by, columns bx / threadIdx.x, so no element index is divided; when the rows
// need no padding (ld == cols) and the source is 16-byte aligned, whole float4s move instead.
__device__ __forceinline__ void split_rows_part(const float *__restrict__ src, float *__restrict__ hi,
                                                float *__restrict__ lo, int64_t rows, int64_t cols, int64_t ld,
                                                unsigned bx, unsigned by, unsigned gx, unsigned gy) {
  if (ld == cols && !(reinterpret_cast<uintptr_t>(src) & 15) && (cols & 3) == 0) {
    const int64_t n4 = rows * cols / 4;
    const int64_t stride = (int64_t)gx * gy * blockDim.x;
    for (int64_t i = ((int64_t)by * gx + bx) * blockDim.x + threadIdx.x; i < n4; i += stride) {
      const float4 x = reinterpret_cast<const float4 *>(src)[i];
      const float4 h = make_float4(to_tf32(x.x), to_tf32(x.y), to_tf32(x.z), to_tf32(x.w));
      reinterpret_cast<float4 *>(hi)[i] = h;
      reinterpret_cast<float4 *>(lo)[i] =
          make_float4(to_tf32(x.x - h.x), to_tf32(x.y - h.y), to_tf32(x.z - h.z), to_tf32(x.w - h.w));
    }
    return;
  }
  for (int64_t r = by; r < rows; r += gy)
    for (int64_t c = (int64_t)bx * blockDim.x + threadIdx.x; c < ld; c += (int64_t)gx * blockDim.x) {
      const float x = c < cols ? src[r * cols + c] : 0.0f;
      const float h = to_tf32(x);
      hi[r * ld + c] = h;
      lo[r * ld + c] = to_tf32(x - h);
    }
}

// [nb][K][N] -> [nb][N][ld] hi / lo for one block of 32 K rows x 128 N columns (bx over N, by over
// ld, bz the batch), transposing through a 32 x 129 shared tile; 256 threads. Loads are float4 along
// N when B allows it (16-byte base, N a multiple of 4); each warp then writes 16 output rows, lane =
// k, so every store is one 128-byte row segment and the tile reads are conflict-free.
__device__ __forceinline__ void split_transpose_part(const float *__restrict__ src, float *__restrict__ hi,
                                                     float *__restrict__ lo, int K, int N, int ld, unsigned bx,
                                                     unsigned by, unsigned bz, float (*tile)[129]) {
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int k0 = by * 32, n0 = bx * 128;
  const float *s = src + (int64_t)bz * K * N;
  const bool vec = !(reinterpret_cast<uintptr_t>(src) & 15) && (N & 3) == 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int kr = ty + 8 * i, k = k0 + kr, n = n0 + 4 * tx;
    float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (k < K) {
      if (vec && n + 3 < N) {
        x = *reinterpret_cast<const float4 *>(s + (int64_t)k * N + n);
      } else {
        const float *row = s + (int64_t)k * N;
        if (n < N) x.x = row[n];
        if (n + 1 < N) x.y = row[n + 1];
        if (n + 2 < N) x.z = row[n + 2];
        if (n + 3 < N) x.w = row[n + 3];
      }
    }
    tile[kr][4 * tx] = x.x, tile[kr][4 * tx + 1] = x.y, tile[kr][4 * tx + 2] = x.z, tile[kr][4 * tx + 3] = x.w;
  }
  __syncthreads();
  const int k = k0 + tx;
  if (k >= ld) return;
  float *h = hi + (int64_t)bz * N * ld + k;
  float *l = lo + (int64_t)bz * N * ld + k;
#pragma unroll 4
  for (int r = 0; r < 16; ++r) {
    const int nl = ty * 16 + r, n = n0 + nl;
    if (n < N) {
      const float x = tile[tx][nl];
      const float hv = to_tf32(x);
      h[(int64_t)n * ld] = hv;
      l[(int64_t)n * ld] = to_tf32(x - hv);
    }
  }
}

__global__ void split_prologue_kernel(const SplitJob j) {
  __shared__ float tile[32][129];
  grid_dependents_launch();  // the GEMM may start its set-up now; it waits for this grid's completion
  unsigned blk = blockIdx.x;
  const unsigned na = j.ax * j.ay;
  if (blk < na) {
    split_rows_part(j.a, j.a_hi, j.a_lo, j.a_rows, j.k, j.ld, blk % j.ax, blk / j.ax, j.ax, j.ay);
    return;
  }
  blk -= na;
  const unsigned nbk = j.bx * j.by * j.bz;
  if (blk < nbk) {
    if (j.b_trans) {
      const unsigned bx = blk % j.bx, rest = blk / j.bx;
      split_transpose_part(j.b, j.b_hi, j.b_lo, (int)j.k, j.n, (int)j.ld, bx, rest % j.by, rest / j.by, tile);
    } else {
      split_rows_part(j.b, j.b_hi, j.b_lo, j.b_rows, j.k, j.ld, blk % j.bx, blk / j.bx, j.bx, j.by);
    }
    return;
  }
  blk -= nbk;
  // C: 16-byte stores (C's base is 16-byte aligned: it is written through TMA), a scalar tail
  const int64_t n4 = j.c_floats / 4;
  const int64_t stride = (int64_t)j.cblocks * blockDim.x;
  for (int64_t i = (int64_t)blk * blockDim.x + threadIdx.x; i < n4; i += stride)
    reinterpret_cast<float4 *>(j.c)[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int64_t i = 4 * n4 + (int64_t)blk * blockDim.x + threadIdx.x; i < j.c_floats; i += stride) j.c[i] = 0.0f;
}

// Fills the block ranges of a SplitJob and launches it: a row split moves about four float4s per
// thread when its rows are contiguous (else up to 8 blocks per SM walk the rows), the transpose takes
// one block per 32 x 128 tile, the zeroing of C about four float4s per thread; for 1024^3 the whole
// prologue is one wave of blocks.
static int launch_split_prologue(mpc_device *dev, SplitJob j, cudaStream_t st) {
  const int64_t sms = dev->prop.multiProcessorCount;
  auto clamp_blocks = [sms](int64_t b) { return (unsigned)(b < 1 ? 1 : b < sms * 8 ? b : sms * 8); };
  auto rows_grid = [&](const float *src, int64_t rows, int64_t ld, unsigned &gx, unsigned &gy) {
    if (ld == j.k && !(reinterpret_cast<uintptr_t>(src) & 15) && (j.k & 3) == 0) {  // the flat float4 path
      gx = 1;
      gy = clamp_blocks((rows * ld / 4 + 1023) / 1024);
      return;
    }
    const int64_t x = (ld + 255) / 256 < 8 ? (ld + 255) / 256 : 8;
    const int64_t y = rows < sms * 8 / x ? rows : sms * 8 / x;
    gx = (unsigned)(x > 0 ? x : 1);
    gy = (unsigned)(y > 0 ? y : 1);
  };
  rows_grid(j.a, j.a_rows, j.ld, j.ax, j.ay);
  if (j.b_trans) {
    j.bx = (unsigned)((j.n + 127) / 128), j.by = (unsigned)((j.ld + 31) / 32), j.bz = (unsigned)j.nb;
  } else {
    rows_grid(j.b, j.b_rows, j.ld, j.bx, j.by);
    j.bz = 1;
  }
  j.cblocks = j.c ? clamp_blocks((j.c_floats / 4 + 1023) / 1024) : 0;
  const uint64_t total = (uint64_t)j.ax * j.ay + (uint64_t)j.bx * j.by * j.bz + j.cblocks;
  if (total >= (1ull << 31)) return fail(MPC_ERR_UNSUPPORTED, "gemm: tf32 split prologue of %llu blocks", (unsigned long long)total);
  split_prologue_kernel<<<(unsigned)total, 256, 0, st>>>(j);
  dev->launches++;
  return check_launch(dev, "split_prologue_kernel");
}

// K == 0: C = epilogue(0).
__global__ void fill_epilogue_kernel(void *C, int out_dtype, int64_t rows, int64_t N, const float *bias, int epi) {
  const int64_t total = rows * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    float v = 0.0f;
    if (epi & MPC_EPI_BIAS) v += bias[i % N];
    if (epi & MPC_EPI_GELU) v = gelu_erf_f32(v);
    if (out_dtype == MPC_F32)
      static_cast<float *>(C)[i] = v;
    else if (out_dtype == MPC_BF16)
      static_cast<__nv_bfloat16 *>(C)[i] = __float2bfloat16_rn(v);
    else
      static_cast<__half *>(C)[i] = __float2half_rn(v);
  }
}

template <int KIND, bool B_MN, int BN, int STAGES, int NDST = 1, bool PAIR = false, bool RES16 = false, int EPI_BUFS = 1>
int launch(mpc_device *dev, const MapsT<NDST> &maps, const Params &p, cudaStream_t st) {
  using C = Cfg<KIND, B_MN, BN, STAGES, PAIR, EPI_BUFS>;
  auto kern = gemm_kernel<KIND, B_MN, BN, STAGES, NDST, PAIR, RES16, EPI_BUFS>;
  static bool configured[64] = {};
  static int pairs_resident[64] = {};
  const int ord = dev->ordinal & 63;
  if (!configured[ord]) {
    MPC_CUDA(dev, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    configured[ord] = true;
  }
  if constexpr (PAIR) {
    // One persistent pair per TPC that can hold one: as many clusters of two as fit at once.
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (!pairs_resident[ord]) {
      cfg.gridDim = dim3(2 * (dev->prop.multiProcessorCount / 2));
      int n = 0;
      MPC_CUDA(dev, cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
      if (n < 1) return fail(MPC_ERR_UNSUPPORTED, "gemm_kernel: no CTA pair fits on this device");
      pairs_resident[ord] = n;
    }
    const int pairs = p.tiles_total < pairs_resident[ord] ? p.tiles_total : pairs_resident[ord];
    cfg.gridDim = dim3(2 * pairs);
    MPC_CUDA(dev, cudaLaunchKernelEx(&cfg, kern, maps, p));
  } else if constexpr (KIND == kTF32x3) {
    // Launched programmatically after the split prologue: the set-up (barriers, tensor memory,
    // descriptor prefetch) overlaps the prologue's last blocks; the kernel waits for its planes.
    const int grid = p.tiles_total < dev->prop.multiProcessorCount ? p.tiles_total : dev->prop.multiProcessorCount;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    MPC_CUDA(dev, cudaLaunchKernelEx(&cfg, kern, maps, p));
  } else {
    const int grid = p.tiles_total < dev->prop.multiProcessorCount ? p.tiles_total : dev->prop.multiProcessorCount;
    kern<<<grid, C::THREADS, C::SMEM, st>>>(maps, p);
  }
  dev->launches++;
  return check_launch(dev, "gemm_kernel");
}

}  // namespace gemm

// ---- host entry -----------------------------------------------------------------------------
static CUtensorMapDataType tmap_dtype(int dt) {
  switch (dt) {
    case MPC_F32:
      return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    case MPC_F16:
      return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    default:
      return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  }
}

static inline int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

namespace gemm {

// What the descriptor implies once validated: the batch extent, the number of distinct A / B
// matrices the batch strides reach, and the kernel configuration.
struct Prep {
  int64_t batch = 1, nA = 1, nB = 1;
  bool tf32 = false, b_mn = false;
  bool pair = false;  // CTA pairs: 256 x 256 tiles, two SMs per tile
  int BN = 256;
  int splits = 1;     // 3xTF32: 2 = each 128 x 128 tile's K in two halves, reduce-added into a zeroed C
};

// Validates `d` and fills every kernel parameter that does not depend on the output.
// Returns MPC_OK with prep.batch == 0 (or M / N == 0) when there is nothing to compute.
static int prepare(mpc_device *dev, const mpc_gemm_desc *d, const float *bias, const char *who, Params &p, Prep &pr,
                   bool allow_pair = false, bool c_tma = false) {
  const int64_t M = d->m, N = d->n, K = d->k;
  if (M < 0 || N < 0 || K < 0)
    return fail(MPC_ERR_INVALID, "%s: negative dimension m=%lld n=%lld k=%lld", who, (long long)M, (long long)N,
                (long long)K);
  if (d->dtype_in != MPC_F32 && d->dtype_in != MPC_F16 && d->dtype_in != MPC_BF16)
    return fail(MPC_ERR_INVALID, "%s: dtype_in %d is not f32/f16/bf16", who, d->dtype_in);
  if (d->dtype_out != MPC_F32 && d->dtype_out != MPC_F16 && d->dtype_out != MPC_BF16)
    return fail(MPC_ERR_INVALID, "%s: dtype_out %d is not f32/f16/bf16", who, d->dtype_out);
  if (d->b_layout != MPC_B_KN && d->b_layout != MPC_B_NK) return fail(MPC_ERR_INVALID, "%s: b_layout %d", who, d->b_layout);
  if (d->batch_rank < 0 || d->batch_rank > 4) return fail(MPC_ERR_INVALID, "%s: batch_rank %d", who, d->batch_rank);
  if ((d->epilogue & MPC_EPI_BIAS) && !bias) return fail(MPC_ERR_INVALID, "%s: BIAS epilogue without bias", who);
  if (M > (1 << 30) || N > (1 << 30) || K > (1 << 30)) return fail(MPC_ERR_UNSUPPORTED, "%s: dimension above 2^30", who);
  p = Params{};
  pr = Prep{};
  p.brank = d->batch_rank;
  for (int i = 0; i < d->batch_rank; ++i) {
    const int64_t sz = d->batch_shape[i];
    if (sz < 0) return fail(MPC_ERR_INVALID, "%s: batch_shape[%d] = %lld", who, i, (long long)sz);
    pr.batch *= sz;
    const int64_t sa = d->a_batch_stride[i], sb = d->b_batch_stride[i];
    if (sa < 0 || sb < 0 || (M * K && sa % (M * K)) || (K * N && sb % (K * N)))
      return fail(MPC_ERR_INVALID, "%s: batch strides must be whole matrices (axis %d: %lld, %lld)", who, i,
                  (long long)sa, (long long)sb);
    p.bshape[i] = (int)sz;
    p.a_bstride[i] = M * K ? (int)(sa / (M * K)) : 0;
    p.b_bstride[i] = K * N ? (int)(sb / (K * N)) : 0;
    if (sz > 0) {
      pr.nA += (sz - 1) * p.a_bstride[i];
      pr.nB += (sz - 1) * p.b_bstride[i];
    }
  }
  pr.tf32 = d->dtype_in == MPC_F32;
  pr.b_mn = !pr.tf32 && d->b_layout == MPC_B_KN;
  pr.BN = pr.tf32 ? 128 : 256;
  // 3xTF32 on a problem with fewer 128 x 128 tiles than SMs: the two K halves of each tile on two SMs
  // (f32 C written through TMA, no GELU / residual, at least 8 K blocks per tile: the halves add into
  // a zeroed C, and with two addends the sum is the same whichever lands first), else 128 x 64 tiles.
  const int64_t tiles128 = pr.batch * ((M + 127) / 128) * ((N + 127) / 128);
  if (pr.tf32 && tiles128 < dev->prop.multiProcessorCount) {
    if (c_tma && d->dtype_out == MPC_F32 && !(d->epilogue & (MPC_EPI_GELU | MPC_EPI_RESIDUAL)) && (K + 31) / 32 >= 8 &&
        2 * tiles128 <= dev->prop.multiProcessorCount)
      pr.splits = 2;
    else
      pr.BN = 64;
  }
  // f16 / bf16 with at least one 256 x 256 tile per resident pair: CTA pairs (half the B bytes
  // per SM, a third less operand traffic per product than 128 x 256 tiles on one SM).
  pr.pair = allow_pair && !pr.tf32 &&
            pr.batch * ((M + 255) / 256) * ((N + 255) / 256) >= dev->prop.multiProcessorCount / 2;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.tiles_m = (int)((M + (pr.pair ? 255 : 127)) / (pr.pair ? 256 : 128));
  p.tiles_n = (int)((N + pr.BN - 1) / pr.BN);
  const int64_t tiles = pr.batch * p.tiles_m * p.tiles_n * pr.splits;
  if (tiles > INT32_MAX) return fail(MPC_ERR_UNSUPPORTED, "%s: %lld tiles", who, (long long)tiles);
  p.tiles_total = (int)tiles;  // work units: tiles x K splits
  p.k_blocks = (int)((K + (pr.tf32 ? 31 : 63)) / (pr.tf32 ? 32 : 64));
  p.splits = pr.splits;
  p.kb_split = (p.k_blocks + pr.splits - 1) / pr.splits;
  p.group_m = 16;
  p.alpha = d->alpha;
  p.bias = bias;
  p.epilogue = d->epilogue & (MPC_EPI_BIAS | MPC_EPI_GELU | MPC_EPI_RESIDUAL);
  p.idesc = make_idesc(pr.tf32 ? kFmtTF32 : (d->dtype_in == MPC_BF16 ? kFmtBF16 : kFmtF16), pr.b_mn,
                       pr.pair ? 256 : 128, pr.BN);
  p.out_dtype = d->dtype_out;
  p.err = dev->d_err;
  p.timeout_ns = dev->timeout_ns;
  p.ndst = 1;
  return MPC_OK;
}

// Operand scratch: tf32 hi / lo planes, or pitch-padded copies of misaligned half operands.
struct OperandScratch {
  Scratch a, b, a2, b2;
};

// Builds the A / B maps (and runs the tf32 split prologue or the padding copies they need). c_zero:
// C, for the split prologue to zero (split-K halves add into it), or null.
template <int NDST>
static int operand_maps(mpc_device *dev, const mpc_gemm_desc *d, const Prep &pr, const void *A, const void *B,
                        MapsT<NDST> &maps, OperandScratch &s, cudaStream_t st, float *c_zero = nullptr,
                        int64_t c_floats = 0) {
  const int64_t M = d->m, N = d->n, K = d->k, nA = pr.nA, nB = pr.nB;
  const CUtensorMapSwizzle SW = CU_TENSOR_MAP_SWIZZLE_128B;
  int rc;
  if (pr.tf32) {
    const int64_t ldk = round_up(K, 4);
    if ((rc = s.a.get(dev, st, (size_t)(nA * M * ldk) * 4)) || (rc = s.a2.get(dev, st, (size_t)(nA * M * ldk) * 4)) ||
        (rc = s.b.get(dev, st, (size_t)(nB * N * ldk) * 4)) || (rc = s.b2.get(dev, st, (size_t)(nB * N * ldk) * 4)))
      return rc;
    SplitJob j = {};
    j.a = static_cast<const float *>(A), j.a_hi = (float *)s.a.ptr, j.a_lo = (float *)s.a2.ptr, j.a_rows = nA * M;
    j.b = static_cast<const float *>(B), j.b_hi = (float *)s.b.ptr, j.b_lo = (float *)s.b2.ptr, j.b_rows = nB * N;
    j.b_trans = d->b_layout == MPC_B_NK ? 0 : 1, j.nb = (int)nB, j.n = (int)N, j.k = K, j.ld = ldk;
    j.c = c_zero, j.c_floats = c_zero ? c_floats : 0;
    if ((rc = launch_split_prologue(dev, j, st))) return rc;
    const CUtensorMapDataType f32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    if ((rc = make_map_3d(&maps.a, f32, s.a.ptr, K, M, nA, ldk * 4, M * ldk * 4, 32, 128, SW)) ||
        (rc = make_map_3d(&maps.a_lo, f32, s.a2.ptr, K, M, nA, ldk * 4, M * ldk * 4, 32, 128, SW)) ||
        (rc = make_map_3d(&maps.b, f32, s.b.ptr, K, N, nB, ldk * 4, N * ldk * 4, 32, pr.BN, SW)) ||
        (rc = make_map_3d(&maps.b_lo, f32, s.b2.ptr, K, N, nB, ldk * 4, N * ldk * 4, 32, pr.BN, SW)))
      return rc;
    return MPC_OK;
  }
  const size_t es = 2;
  const CUtensorMapDataType dt = tmap_dtype(d->dtype_in);
  // A: [nA][M][K]; a padded copy when K*2 bytes is not a multiple of 16 or A is misaligned.
  const void *ap = A;
  int64_t lda = K;
  if (((uintptr_t)A & 15) || (K * es) % 16) {
    lda = round_up(K, 8);
    if ((rc = s.a.get(dev, st, (size_t)(nA * M * lda) * es))) return rc;
    MPC_CUDA(dev, cudaMemcpy2DAsync(s.a.ptr, lda * es, A, K * es, K * es, nA * M, cudaMemcpyDeviceToDevice, st));
    ap = s.a.ptr;
  }
  if ((rc = make_map_3d(&maps.a, dt, ap, K, M, nA, lda * es, M * lda * es, 64, 128, SW))) return rc;
  const void *bp = B;
  if (pr.b_mn) {  // B [nB][K][N]
    int64_t ldb = N;
    if (((uintptr_t)B & 15) || (N * es) % 16) {
      ldb = round_up(N, 8);
      if ((rc = s.b.get(dev, st, (size_t)(nB * K * ldb) * es))) return rc;
      MPC_CUDA(dev, cudaMemcpy2DAsync(s.b.ptr, ldb * es, B, N * es, N * es, nB * K, cudaMemcpyDeviceToDevice, st));
      bp = s.b.ptr;
    }
    return make_map_3d(&maps.b, dt, bp, N, K, nB, ldb * es, K * ldb * es, 64, 64, SW);
  }
  int64_t ldb = K;  // B [nB][N][K]
  if (((uintptr_t)B & 15) || (K * es) % 16) {
    ldb = round_up(K, 8);
    if ((rc = s.b.get(dev, st, (size_t)(nB * N * ldb) * es))) return rc;
    MPC_CUDA(dev, cudaMemcpy2DAsync(s.b.ptr, ldb * es, B, K * es, K * es, nB * N, cudaMemcpyDeviceToDevice, st));
    bp = s.b.ptr;
  }
  return make_map_3d(&maps.b, dt, bp, K, N, nB, ldb * es, N * ldb * es, 64, pr.pair ? 128 : 256, SW);
}

}  // namespace gemm

int gemm_run(mpc_device *dev, const mpc_gemm_desc *d, const void *A, const void *B, void *Cout, const float *bias,
             const void *resid, cudaStream_t st) {
  using namespace gemm;
  Params p;
  Prep pr;
  const bool c_tma = !((uintptr_t)Cout & 15) && (d->n * (int64_t)dtype_size(d->dtype_out)) % 16 == 0;
  int rc = prepare(dev, d, bias, "mpc_gemm", p, pr, true, c_tma);
  if (rc) return rc;
  const int64_t M = d->m, N = d->n, K = d->k, batch = pr.batch;
  if ((d->epilogue & MPC_EPI_RESIDUAL) && !resid)
    return fail(MPC_ERR_INVALID, "mpc_gemm: RESIDUAL epilogue without a residual matrix");
  if (batch == 0 || M == 0 || N == 0) return MPC_OK;
  if (!A || !B || !Cout) return fail(MPC_ERR_INVALID, "mpc_gemm: null operand pointer");
  const size_t eo = dtype_size(d->dtype_out);
  p.resid = (d->epilogue & MPC_EPI_RESIDUAL) ? resid : nullptr;
  p.resid_vec = p.resid && !((uintptr_t)resid & 15) && (N * eo) % 16 == 0;
  if (K == 0 && p.resid)
    return fail(MPC_ERR_UNSUPPORTED, "mpc_gemm: RESIDUAL epilogue with K == 0");
  if (K == 0) {
    gemm::fill_epilogue_kernel<<<1184, 256, 0, st>>>(Cout, d->dtype_out, batch * M, N, bias, d->epilogue);
    dev->launches++;
    return check_launch(dev, "fill_epilogue_kernel");
  }
  Maps maps;
  memset(&maps, 0, sizeof(maps));
  OperandScratch s;
  // Output: TMA stores when the rows are 16-byte aligned; otherwise the epilogue writes the staged
  // blocks with plain stores (the element alignment suffices) and the map is unused.
  void *cdst = Cout;
  int64_t ldc = N;
  if (((uintptr_t)Cout & 15) || (N * eo) % 16) {
    if ((uintptr_t)Cout % eo) return fail(MPC_ERR_INVALID, "mpc_gemm: C is not aligned to its element size");
    p.c_direct = Cout;
    ldc = round_up(N, 16 / eo);  // any valid map: it is never used
  }
  if (p.c_direct) cdst = reinterpret_cast<void *>((uintptr_t)Cout & ~uintptr_t(15));  // aligned; never stored to
  if ((rc = make_map_3d(&maps.c[0], tmap_dtype(d->dtype_out), cdst, N, M, batch, ldc * eo, M * ldc * eo,
                        128 / (uint32_t)eo, 32, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  // split K: the two halves of each tile add into C, which the split prologue zeroes
  if ((rc = operand_maps(dev, d, pr, A, B, maps, s, st, pr.splits > 1 ? static_cast<float *>(Cout) : nullptr,
                         batch * M * N)))
    return rc;
  const bool res16 = (p.epilogue & MPC_EPI_RESIDUAL) && !(p.epilogue & MPC_EPI_GELU) && eo == 2 && p.resid_vec;
  if (pr.tf32 && pr.BN == 64)
    rc = launch<kTF32x3, false, 64, 4>(dev, maps, p, st);
  else if (pr.tf32)
    rc = launch<kTF32x3, false, 128, 3>(dev, maps, p, st);
  else if (res16 && pr.pair && pr.b_mn)
    rc = launch<kHalf, true, 256, 6, 1, true, true>(dev, maps, p, st);
  else if (res16 && pr.pair)  // linear on pairs: two staging blocks per epilogue warp
    rc = launch<kHalf, false, 256, 5, 1, true, true, 2>(dev, maps, p, st);
  else if (res16 && pr.b_mn)
    rc = launch<kHalf, true, 256, 4, 1, false, true>(dev, maps, p, st);
  else if (res16)
    rc = launch<kHalf, false, 256, 4, 1, false, true>(dev, maps, p, st);
  else if (pr.pair && pr.b_mn)
    rc = launch<kHalf, true, 256, 6, 1, true>(dev, maps, p, st);
  else if (pr.pair)
    rc = launch<kHalf, false, 256, 5, 1, true, false, 2>(dev, maps, p, st);
  else if (pr.b_mn)
    rc = launch<kHalf, true, 256, 4>(dev, maps, p, st);
  else
    rc = launch<kHalf, false, 256, 4>(dev, maps, p, st);
  return rc;
}

int gemm_capabilities(mpc_device *dev, mpc_gemm_caps *c) {
  memset(c, 0, sizeof(*c));
  // The conditions prepare() applies when it picks a kernel, reported rather than re-derived.
  c->f16 = c->bf16 = c->f32_3xtf32 = 1;
  c->cta_pairs = dev->prop.major == 10 ? 1 : 0;
  c->sm_count = dev->prop.multiProcessorCount;
  c->pair_min_tiles = dev->prop.multiProcessorCount / 2;
  c->tf32_narrow_below = dev->prop.multiProcessorCount;
  c->attention_tc_head_dims = 1 | 2;
  c->attention_max_head_dim = 256;
  c->max_dim = int64_t(1) << 30;
  return MPC_OK;
}

// The product stored into several row-major matrices at once (row pitch ldc elements, columns
// col_offset .. col_offset + N - 1 of each): the epilogue issues one TMA store per destination for
// every output block. With the destinations being every rank's copy of a column-split result in
// peer memory, this is a GEMM fused with its all-gather.
int gemm_run_multi(mpc_device *dev, const mpc_gemm_desc *d, const void *A, const void *B, const float *bias,
                   void *const *dsts, int ndst, int64_t ldc, int64_t col_offset, cudaStream_t st) {
  using namespace gemm;
  const char *who = "mpc_gemm_multi_store";
  if (ndst < 1 || ndst > kMaxDst) return fail(MPC_ERR_INVALID, "%s: %d destinations (1..%d)", who, ndst, kMaxDst);
  if (!dsts) return fail(MPC_ERR_INVALID, "%s: null destination list", who);
  Params p;
  Prep pr;
  // CTA pairs only for a single destination: with peer destinations (the all-gather fused into
  // the epilogue) the paired kernel measured 6-8% slower on two GPUs than 128 x 256 tiles on one SM.
  int rc = prepare(dev, d, bias, who, p, pr, ndst == 1);
  if (rc) return rc;
  if (pr.tf32) return fail(MPC_ERR_UNSUPPORTED, "%s: f16 / bf16 operands only", who);
  if (d->epilogue & MPC_EPI_RESIDUAL) return fail(MPC_ERR_UNSUPPORTED, "%s: no RESIDUAL epilogue", who);
  const int64_t M = d->m, N = d->n, K = d->k, batch = pr.batch;
  const size_t eo = dtype_size(d->dtype_out);
  if (col_offset < 0 || ldc < col_offset + N)
    return fail(MPC_ERR_INVALID, "%s: columns [%lld, %lld) do not fit rows of %lld", who, (long long)col_offset,
                (long long)(col_offset + N), (long long)ldc);
  if ((ldc * eo) % 16 || (col_offset * eo) % 16)
    return fail(MPC_ERR_INVALID, "%s: row pitch and column offset must be multiples of 16 bytes", who);
  for (int i = 0; i < ndst; ++i)
    if (!dsts[i] || ((uintptr_t)dsts[i] & 15)) return fail(MPC_ERR_INVALID, "%s: destination %d null or misaligned", who, i);
  if (batch == 0 || M == 0 || N == 0) return MPC_OK;
  if (!A || !B) return fail(MPC_ERR_INVALID, "%s: null operand pointer", who);
  if (K == 0) return fail(MPC_ERR_UNSUPPORTED, "%s: K == 0", who);
  MapsT<kMaxDst> maps;
  memset(&maps, 0, sizeof(maps));
  for (int i = 0; i < ndst; ++i) {
    void *base = static_cast<uint8_t *>(dsts[i]) + col_offset * eo;
    if ((rc = make_map_3d(&maps.c[i], tmap_dtype(d->dtype_out), base, N, M, batch, ldc * eo, M * ldc * eo,
                          128 / (uint32_t)eo, 32, CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
  }
  p.ndst = ndst;
  OperandScratch s;
  if ((rc = operand_maps(dev, d, pr, A, B, maps, s, st))) return rc;
  if (pr.pair && pr.b_mn) return launch<kHalf, true, 256, 6, kMaxDst, true>(dev, maps, p, st);
  if (pr.pair) return launch<kHalf, false, 256, 6, kMaxDst, true>(dev, maps, p, st);
  if (pr.b_mn) return launch<kHalf, true, 256, 4, kMaxDst>(dev, maps, p, st);
  return launch<kHalf, false, 256, 4, kMaxDst>(dev, maps, p, st);
}

// ---------------------------------------------------------------------------------------------
// Allocation-free f32 GEMM (3xTF32) for callers that cannot allocate device memory.
//
// Some callers of this library may not call cudaMalloc: a host runtime that hands the library a
// fixed, pre-sized memory budget, or a caller whose own allocator owns every device byte.
// mpc_gemm's f32 path needs scratch memory for the tf32 hi / lo planes of A and B (and a
// pitch-padded copy of C when C's rows are not 16-byte aligned), which it takes from the device
// allocator. mpc_gemm_f32_noalloc runs the same kernels with that scratch in one file-scope device
// array instead: it allocates nothing and needs no mpc_device handle, working on the calling
// thread's current CUDA device and the given stream.
//
// The array is kNoAllocScratchBytes (32 MiB) plus a 256-byte header holding the kernels' error
// word. Every GPU that loads this library holds it until the process exits. All calls share it
// and it keeps the last call's contents: each call rewrites every scratch byte it reads, but two
// calls whose work overlaps on the GPU (different streams, or no ordering between them) race on the
// array; serialise them. The first call on a device sets up that device (it resolves the array's
// device address with cudaGetSymbolAddress and reads the device properties); make that first call
// before any stream capture. The set-up is not redone after cudaDeviceReset. A kernel-side wait that
// runs out leaves its site in the error word, which later calls keep (no call clears it):
// mpc_gemm_f32_noalloc_status reads it and clears it.
// ---------------------------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
constexpr size_t kNoAllocHeader = 256;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocHeader + kNoAllocScratchBytes];

struct NoAllocDevice {
  std::once_flag once;
  int status = MPC_OK;
  unsigned char *base = nullptr;  // device address of g_noalloc_scratch on this device
  mpc_device lite;                // ordinal, properties and error word for the shared launch code
};
NoAllocDevice g_noalloc[64];

// The calling thread's current device, set up once (see above).
int noalloc_device(const char *who, NoAllocDevice **out) {
  int ord = -1;
  cudaError_t e = cudaGetDevice(&ord);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, who);
  if (ord < 0 || ord >= 64) return fail(MPC_ERR_UNSUPPORTED, "%s: device ordinal %d", who, ord);
  NoAllocDevice &nd = g_noalloc[ord];
  std::call_once(nd.once, [&] {
    void *p = nullptr;
    cudaError_t r = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // with device `ord` current
    if (r == cudaSuccess) r = cudaGetDeviceProperties(&nd.lite.prop, ord);
    if (r != cudaSuccess) {
      nd.status = cuda_fail(nullptr, r, "mpc_gemm_f32_noalloc: device set-up");
      return;
    }
    nd.base = static_cast<unsigned char *>(p);
    nd.lite.ordinal = ord;
    nd.lite.d_err = reinterpret_cast<int *>(nd.base);
  });
  if (nd.status != MPC_OK) return fail(nd.status, "%s: set-up of device %d failed earlier", who, ord);
  *out = &nd;
  return MPC_OK;
}
}  // namespace
}  // namespace mpc

extern "C" int mpc_gemm_f32_noalloc(const mpc_gemm_desc *d, const float *A, const float *B, float *Cout,
                                    const float *bias, mpc_stream s) {
  using namespace mpc;
  using namespace mpc::gemm;
  const char *who = "mpc_gemm_f32_noalloc";
  NoAllocDevice *nd = nullptr;
  int rc = noalloc_device(who, &nd);
  if (rc) return rc;
  if (!d) return fail(MPC_ERR_INVALID, "%s: null descriptor", who);
  if (d->dtype_in != MPC_F32 || d->dtype_out != MPC_F32)
    return fail(MPC_ERR_INVALID, "%s: f32 inputs and output only (got %d -> %d)", who, d->dtype_in, d->dtype_out);
  if (d->epilogue & MPC_EPI_RESIDUAL) return fail(MPC_ERR_UNSUPPORTED, "%s: no RESIDUAL epilogue", who);
  mpc_device *dev = &nd->lite;
  Params p;
  Prep pr;
  // The same validation and kernel choice as mpc_gemm's f32 path (tile limits, the 128 x 64 tiles
  // for problems with fewer 128 x 128 tiles than SMs).
  if ((rc = prepare(dev, d, bias, who, p, pr, false, true))) return rc;  // C goes out through TMA (staged if need be)
  const int64_t M = d->m, N = d->n, K = d->k, batch = pr.batch;
  if (batch == 0 || M == 0 || N == 0) return MPC_OK;
  if (!A || !B || !Cout) return fail(MPC_ERR_INVALID, "%s: null operand pointer", who);
  // Scratch layout: A_hi | A_lo | B_hi | B_lo (K pitch rounded to 4 floats), then C staging.
  const int64_t ldk = round_up(K, 4);
  const bool stage_c = ((uintptr_t)Cout & 15) || (N % 4);
  const int64_t ldc = stage_c ? round_up(N, 4) : N;
  const size_t a_plane = (size_t)(pr.nA * M * ldk) * 4, b_plane = (size_t)(pr.nB * N * ldk) * 4;
  const size_t need = 2 * a_plane + 2 * b_plane + (stage_c ? (size_t)(batch * M * ldc) * 4 : 0);
  if (K > 0 && need > kNoAllocScratchBytes)
    return fail(MPC_ERR_INVALID,
                "%s: needs %zu bytes of scratch, above its %zu-byte static maximum (use mpc_gemm for this size)", who,
                need, kNoAllocScratchBytes);
  cudaStream_t st = static_cast<cudaStream_t>(s);
  if (K == 0) {
    fill_epilogue_kernel<<<1184, 256, 0, st>>>(Cout, MPC_F32, batch * M, N, bias, d->epilogue);
    return check_launch(dev, "fill_epilogue_kernel");
  }
  unsigned char *scratch = nd->base + kNoAllocHeader;
  float *a_hi = reinterpret_cast<float *>(scratch), *a_lo = reinterpret_cast<float *>(scratch + a_plane);
  float *b_hi = reinterpret_cast<float *>(scratch + 2 * a_plane);
  float *b_lo = reinterpret_cast<float *>(scratch + 2 * a_plane + b_plane);
  float *cdst = stage_c ? reinterpret_cast<float *>(scratch + 2 * a_plane + 2 * b_plane) : Cout;
  SplitJob j = {};
  j.a = A, j.a_hi = a_hi, j.a_lo = a_lo, j.a_rows = pr.nA * M;
  j.b = B, j.b_hi = b_hi, j.b_lo = b_lo, j.b_rows = pr.nB * N;
  j.b_trans = d->b_layout == MPC_B_NK ? 0 : 1, j.nb = (int)pr.nB, j.n = (int)N, j.k = K, j.ld = ldk;
  j.c = pr.splits > 1 ? cdst : nullptr;  // the two K halves of each tile add into it
  j.c_floats = batch * M * ldc;
  if ((rc = launch_split_prologue(dev, j, st))) return rc;
  Maps maps;
  memset(&maps, 0, sizeof(maps));
  const CUtensorMapDataType f32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const CUtensorMapSwizzle SW = CU_TENSOR_MAP_SWIZZLE_128B;
  if ((rc = make_map_3d(&maps.a, f32, a_hi, K, M, pr.nA, ldk * 4, M * ldk * 4, 32, 128, SW)) ||
      (rc = make_map_3d(&maps.a_lo, f32, a_lo, K, M, pr.nA, ldk * 4, M * ldk * 4, 32, 128, SW)) ||
      (rc = make_map_3d(&maps.b, f32, b_hi, K, N, pr.nB, ldk * 4, N * ldk * 4, 32, pr.BN, SW)) ||
      (rc = make_map_3d(&maps.b_lo, f32, b_lo, K, N, pr.nB, ldk * 4, N * ldk * 4, 32, pr.BN, SW)) ||
      (rc = make_map_3d(&maps.c[0], f32, cdst, N, M, batch, ldc * 4, M * ldc * 4, 32, 32, SW)))
    return rc;
  rc = pr.BN == 64 ? launch<kTF32x3, false, 64, 4>(dev, maps, p, st) : launch<kTF32x3, false, 128, 3>(dev, maps, p, st);
  if (rc) return rc;
  if (stage_c)
    MPC_CUDA(dev, cudaMemcpy2DAsync(Cout, N * 4, cdst, ldc * 4, N * 4, batch * M, cudaMemcpyDeviceToDevice, st));
  return MPC_OK;
}

extern "C" int mpc_gemm_f32_noalloc_status(mpc_stream s) {
  using namespace mpc;
  const char *who = "mpc_gemm_f32_noalloc_status";
  NoAllocDevice *nd = nullptr;
  int rc = noalloc_device(who, &nd);
  if (rc) return rc;
  MPC_CUDA(nullptr, cudaStreamSynchronize(static_cast<cudaStream_t>(s)));
  int word = 0;
  MPC_CUDA(nullptr, cudaMemcpy(&word, nd->lite.d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (word == 0) return MPC_OK;
  MPC_CUDA(nullptr, cudaMemset(nd->lite.d_err, 0, sizeof(int)));
  return fail(MPC_ERR_TIMEOUT,
              "%s: a kernel's bounded wait (site 0x%x) ran out in an earlier mpc_gemm_f32_noalloc call on device %d; "
              "that call's output is incomplete",
              who, word, nd->lite.ordinal);
}

extern "C" int mpc_gemm_f32_noalloc_selftest(uint64_t timeout_ns, mpc_stream s) {
  using namespace mpc;
  const char *who = "mpc_gemm_f32_noalloc_selftest";
  if (timeout_ns == 0 || timeout_ns > 10000000000ull) return fail(MPC_ERR_INVALID, "%s: timeout must be in (0, 10 s]", who);
  NoAllocDevice *nd = nullptr;
  int rc = noalloc_device(who, &nd);
  if (rc) return rc;
  return wait_probe_run(&nd->lite, timeout_ns, static_cast<cudaStream_t>(s));
}
