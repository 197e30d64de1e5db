// Fused scaled-dot-product attention, sm_100a: softmax(scale·Q·Kᵀ + mask)·V without materialising
// the score matrix. Replaces Backend.sdpa (packages/tensor-cpu/src/index.ts:821-840), whose CPU
// path builds the full Lq x Lk f64 score panel per head (packages/tensor-core/src/nn-kernels.ts:179-239).
//
// Tensor-core path (f16 / bf16, head dim 64 or 128, 16-byte aligned operands):
//   persistent CTAs (at most one per SM) walk units of (batch, head, 256 query rows) = two 128-row
//   Q tiles sharing every K/V tile, in pairs of a heavy and a light causal q-block so that every
//   pair is the same work. Across units the producer loads the next Q as soon as the last QK has
//   read the current one, and the next unit's QK products overlap the current output; 12 warps:
//   warps 0-3 / 4-7  online softmax of Q tile 0 / 1, one thread per query row: tcgen05.ld the S row,
//                    scale (folded with log2 e), mask, row max, exp2, row sum; P (same type as V) is
//                    tcgen05.st'd back over the first half of the S columns; the O accumulator is
//                    rescaled in TMEM only when a row max grows by more than 2^8 (lazy rescale)
//   warp 8           TMA producer: Q once, then K_j / V_j through a 5-slot shared-memory ring
//   warp 9           one thread issues tcgen05.mma: S_t = Q_t·K_jᵀ (SS, both K-major) and
//                    O_t += P_t·V_j (A = P from TMEM, B = V MN-major); owns the TMEM allocation
//   warps 10-11      idle (they complete the load / MMA warpgroup for register reconfiguration)
//   issue order per KV tile j: QK(1,j), PV(0,j), QK(0,j+1), PV(1,j), so each Q tile's softmax runs
//   while the tensor core works on the other tile. For causal launches over at most 1024 keys
//   (1536 at head dim 64) warp 10 issues Q tile 1's MMAs and warp 9 only tile 0's, each in its
//   own order QK(t,j), PV(t,j), QK(t,j+1). Causal: KV tiles past a Q tile's diagonal are skipped,
//   only diagonal tiles are masked element-wise.
//   TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [256+D,256+2D).
// Generic path (any head dim <= 256, f32 / f16 / bf16, any alignment): one warp per query row on the
// CUDA cores, online softmax in f32 — the role of backend-webgpu's generic sdpa kernel.
#include <algorithm>
#include <cfloat>
#include <vector>

#include "mpc_internal.h"
#include "sm100.cuh"

namespace mpc {
namespace attn {

struct Params {
  int B, H, Hk, Lq, Lk, D;
  int rep;       // H / Hk
  int q_blocks;  // ceil(Lq / 256)
  int n_units;  // B * H * q_blocks
  int causal;
  float scale_log2;  // scale * log2(e)
  int mask_kind;
  const void *mask;
  long long ms[4];
  void *out;
  long long os[3];  // element strides of O's (batch, head, row) axes
  float *lse;
  int dtype;
  int q_pos, k_pos, v_pos;  // map axis (1..3) of head, row, batch: bits 0-1, 2-3, 4-5
  uint32_t idesc_qk, idesc_pv;
  int *err;
  unsigned long long timeout_ns;
};

struct Maps {
  CUtensorMap q, k, v;
};

template <int D>
struct Cfg {
  static constexpr int NSUB = D / 64;             // 128-byte (64-element) column blocks of a head row
  static constexpr int TILE = 128 * D * 2;        // bytes of one 128-row Q, K or V tile
  static constexpr int SUB = 128 * 128;           // bytes of one 128-row x 64-column block
  static constexpr int SLOTS = D == 128 ? 5 : 8;  // K/V ring depth: 2.5 (D=128) or 4 KV tiles ahead
  static constexpr int SMEM = 1024 + 2 * TILE + SLOTS * TILE + 256;
  static constexpr int THREADS = 384;  // 3 warpgroups: softmax 0, softmax 1, load / MMA
  static_assert(SMEM <= 232448, "shared memory budget");
};

__host__ __device__ __forceinline__ int last_kv(const Params &p, int q0t) {
  // Last KV tile any row of the Q tile starting at q0t may see.
  int last_key = p.Lk - 1;
  if (p.causal) last_key = min(last_key, min(q0t + 127, p.Lq - 1));
  return last_key < 0 ? -1 : last_key / 128;
}

__device__ __forceinline__ float mask_add(const Params &p, int b, int h, int q, int k) {
  const long long off = b * p.ms[0] + h * p.ms[1] + q * p.ms[2] + k * p.ms[3];
  if (p.mask_kind == MPC_MASK_BOOL) return static_cast<const uint8_t *>(p.mask)[off] ? 0.0f : -INFINITY;
  return static_cast<const float *>(p.mask)[off] * 1.4426950408889634f;
}

// One unit of work: 256 query rows (two 128-row Q tiles) of one (batch, head).
struct Unit {
  int bh, b, h, kvh, q0;  // kvh: the K/V head within the batch entry
  bool valid1;
  int last0, last1, n_kv;
};

// The k-th unit of this CTA. Pairs (SNAKE false): units are numbered head-major; within a head the
// q-blocks alternate heavy and light (QB-1, 0, QB-2, 1, ...), and each CTA takes units in pairs
// (2i, 2i+1), so under a causal mask every pair carries the same work (head-major order keeps a
// head's K / V in L2). Snake (SNAKE true, chosen by the host under a causal mask when the pairs do
// not divide evenly over the CTAs): units sorted by work, heaviest first (the last q-blocks of
// every head, then the ones before), dealt to the CTAs in rounds that alternate direction, so the
// CTAs' sums stay within about one unit of each other. Returns false past the last unit.
template <bool SNAKE>
__device__ __forceinline__ bool unit_of(const Params &p, int k, Unit &w) {
  // 32-bit arithmetic: the host keeps 2 * n_units + 2 * gridDim.x below 2^31.
  const unsigned qbn = (unsigned)p.q_blocks;
  int qb;
  if constexpr (SNAKE) {
    const unsigned n = (unsigned)k * gridDim.x + ((k & 1) ? gridDim.x - 1 - blockIdx.x : blockIdx.x);
    if (n >= (unsigned)p.n_units) return false;
    const unsigned bhn = (unsigned)p.n_units / qbn;
    const unsigned cls = n / bhn;
    w.bh = (int)(n - cls * bhn);
    qb = (int)(qbn - 1 - cls);
  } else {
    const unsigned u = 2u * (blockIdx.x + (unsigned)(k >> 1) * gridDim.x) + (unsigned)(k & 1);
    if (u >= (unsigned)p.n_units) return false;
    w.bh = (int)(u / qbn);
    const int r = (int)(u - (unsigned)w.bh * qbn);
    qb = (r & 1) ? (r >> 1) : (int)qbn - 1 - (r >> 1);
  }
  w.b = w.bh / p.H;
  w.h = w.bh - w.b * p.H;
  w.kvh = w.h / p.rep;
  w.q0 = qb * 256;
  w.valid1 = w.q0 + 128 < p.Lq;
  w.last0 = last_kv(p, w.q0);
  w.last1 = w.valid1 ? last_kv(p, w.q0 + 128) : -1;
  w.n_kv = max(w.last0, w.last1) + 1;
  return true;
}

// One 128-row tile of a Q / K / V map: the map's outer axes are (head, row, batch) in the order
// `pos` gives (sorted by stride on the host).
__device__ __forceinline__ void load_rows(const CUtensorMap *map, uint64_t *bar, void *dst, int col, int head, int row,
                                          int batch, int pos) {
  const int ph = pos & 3, pr = (pos >> 2) & 3;
  const int c1 = ph == 1 ? head : pr == 1 ? row : batch;
  const int c2 = ph == 2 ? head : pr == 2 ? row : batch;
  const int c3 = ph == 3 ? head : pr == 3 ? row : batch;
  tma_load_4d(map, bar, dst, col, c1, c2, c3);
}

// BF: bf16 operands (P is packed as bf16), else f16. A template parameter, not a run-time flag, so
// that the softmax's inner loops carry no per-element branch on the type.
template <int D, bool BF, bool SNAKE, bool DUAL>
__global__ void __launch_bounds__(384, 1) attn_kernel(const __grid_constant__ Maps maps, const Params p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sq = smem;                 // Q tile 0, Q tile 1
  uint8_t *skv = smem + 2 * C::TILE;  // ring of SLOTS K/V tiles
  uint64_t *bars = reinterpret_cast<uint64_t *>(skv + C::SLOTS * C::TILE);
  uint64_t *q_full = bars;
  uint64_t *q_empty = bars + 1;
  uint64_t *kv_full = bars + 2;
  uint64_t *kv_empty = kv_full + C::SLOTS;
  uint64_t *s_ready = kv_empty + C::SLOTS;  // [2]
  uint64_t *p_ready = s_ready + 2;          // [2]
  uint64_t *o_ready = p_ready + 2;          // [2]
  uint64_t *o_free = o_ready + 2;           // [2]
  uint64_t *drain = o_free + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // DUAL: each Q tile's MMAs come from their own thread (warps 9 and 10), so that one tile's QK and
  // PV follow its own softmax instead of waiting in one in-order stream behind the other tile's,
  // and a tile that finishes a unit early moves on to the next one. The host picks it for causal
  // launches over at most 1024 keys (1536 at head dim 64), where unit boundaries are frequent or
  // the softmax dominates; over longer or non-causal rows the single stream measured faster.
  constexpr bool kDualIssue = DUAL;
  constexpr int kIssuers = kDualIssue ? 2 : 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, kIssuers);
    for (int s = 0; s < C::SLOTS; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], kIssuers);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_ready[t], 1);
      mbar_init(&p_ready[t], 4);
      mbar_init(&o_ready[t], 1);
      mbar_init(&o_free[t], 4);
    }
    mbar_init(drain, kIssuers);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Register reconfiguration (at the head of each role's branch): the load / MMA warpgroup
  // gives registers to the two softmax warpgroups, which keep a whole 128-key score row in
  // registers. Launched at 168 per thread (the host checks):
  // 2 x 128 x 208 + 128 x 88 = 64512 = 384 x 168.
  if (warp >= 10 + (kDualIssue ? 1 : 0)) {
    reg_dealloc<88>();  // the warpgroup's spare warps only wait for the end
  } else if (warp == 8) {
    reg_dealloc<88>();
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&maps.q);
      tma_prefetch_desc(&maps.k);
      tma_prefetch_desc(&maps.v);
      int ring = 0, q_loads = 0;
      bool ok = true;
      Unit w;
      for (int k = 0; ok && unit_of<SNAKE>(p, k, w); ++k) {
        // Q of the previous unit is free once its last QK products have run.
        if (k > 0 && !(ok = mbar_wait(q_empty, (k - 1) & 1, abort_flag, p.err, kErrWaitProducer, p.timeout_ns)))
          break;
        const int nq = w.valid1 ? 2 : 1;
        mbar_expect_tx(q_full, nq * C::TILE);
        for (int t = 0; t < nq; ++t)
          for (int s = 0; s < C::NSUB; ++s)
            load_rows(&maps.q, q_full, sq + t * C::TILE + s * C::SUB, s * 64, w.h, w.q0 + 128 * t, w.b, p.q_pos);
        ++q_loads;
        for (int i = 0; i < 2 * w.n_kv; ++i, ++ring) {
          const int slot = ring % C::SLOTS;
          if (!(ok = mbar_wait(&kv_empty[slot], ((ring / C::SLOTS) & 1) ^ 1, abort_flag, p.err, kErrWaitProducer,
                               p.timeout_ns)))
            break;
          const CUtensorMap *map = (i & 1) ? &maps.v : &maps.k;
          mbar_expect_tx(&kv_full[slot], C::TILE);
          for (int s = 0; s < C::NSUB; ++s)
            load_rows(map, &kv_full[slot], skv + slot * C::TILE + s * C::SUB, s * 64, w.kvh, (i >> 1) * 128, w.b,
                      (i & 1) ? p.v_pos : p.k_pos);
        }
      }
      if (!ok) {  // let the copies in flight land before shared memory is released
        volatile int never = 0;
        if (q_loads > 0) mbar_wait(q_full, (q_loads - 1) & 1, &never, p.err, kErrWaitProducer, p.timeout_ns);
        for (int i = ring > C::SLOTS ? ring - C::SLOTS : 0; i < ring; ++i)
          mbar_wait(&kv_full[i % C::SLOTS], (i / C::SLOTS) & 1, &never, p.err, kErrWaitProducer, p.timeout_ns);
      }
    }
  } else if (warp == 9 || (kDualIssue && warp == 10)) {
    if constexpr (kDualIssue) {
      // ---------------- MMA issuers: warp 9 for Q tile 0, warp 10 for Q tile 1 ----------------
      reg_dealloc<88>();
      if (lane == 0) {
        const int t = warp - 9;
        const uint32_t q_addr = smem_u32(sq) + t * C::TILE;
        auto qk = [&](int slot) {
          const uint32_t b0 = smem_u32(skv + slot * C::TILE);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * C::SUB + (kk & 3) * 32;
            mma_f16_ss(tmem + t * 128, make_sdesc(q_addr + off, 16, 1024), make_sdesc(b0 + off, 16, 1024), p.idesc_qk,
                       kk ? 1u : 0u);
          }
        };
        auto pv = [&](int slot, bool first) {
          const uint32_t v0 = smem_u32(skv + slot * C::TILE);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // 128 keys, 16 per MMA; P packs 2 keys per TMEM column
            mma_f16_ts(tmem + 256 + t * D, tmem + t * 128 + kk * 8, make_sdesc(v0 + kk * 2048, C::SUB, 1024),
                       p.idesc_pv, (first && kk == 0) ? 0u : 1u);
        };
        int ring = 0;    // K/V ring items consumed so far (K_j, V_j of every unit in order)
        int pv_cnt = 0;  // PV products issued for this tile (p_ready phases)
        bool ok = true;
        auto wait_item = [&](int i) {
          return mbar_wait(&kv_full[i % C::SLOTS], (i / C::SLOTS) & 1, abort_flag, p.err, kErrWaitConsumer,
                           p.timeout_ns);
        };
        Unit w;
        for (int k = 0; ok && unit_of<SNAKE>(p, k, w); ++k) {
          const int last = t ? w.last1 : w.last0;  // -1 for a missing second tile
          const int base = ring;                   // K_j is ring item base + 2j, V_j item base + 2j + 1
          if (!(ok = mbar_wait(q_full, k & 1, abort_flag, p.err, kErrWaitConsumer, p.timeout_ns))) break;
          for (int j = 0; j < w.n_kv; ++j) {
            const int sk = (base + 2 * j) % C::SLOTS, sv = (base + 2 * j + 1) % C::SLOTS;
            const bool need = j <= last;
            // Every ring item is waited for before it is released, so a release always counts toward
            // the item's own round of the slot (the producer reloads it only after both releases).
            if (!(ok = wait_item(base + 2 * j))) break;
            tc_fence_after();
            if (need) {
              qk(sk);
              tc_commit(&s_ready[t]);
            }
            tc_commit(&kv_empty[sk]);                 // K_j: once this tile's QK has read it
            if (j + 1 == w.n_kv) tc_commit(q_empty);  // Q: once this tile's last QK has run
            if (!(ok = wait_item(base + 2 * j + 1))) break;
            if (need) {
              if (j == 0 && k > 0) {  // O_t still holds the previous unit until its output has been read
                if (!(ok = mbar_wait(&o_free[t], (k - 1) & 1, abort_flag, p.err, kErrWaitSoftmax, p.timeout_ns))) break;
              }
              if (!(ok = mbar_wait(&p_ready[t], pv_cnt & 1, abort_flag, p.err, kErrWaitSoftmax, p.timeout_ns))) break;
              tc_fence_after();
              pv(sv, j == 0);
              tc_commit(&o_ready[t]);
              ++pv_cnt;
            }
            tc_commit(&kv_empty[sv]);  // V_j: once this tile's PV has read it
          }
          ring = base + 2 * w.n_kv;
        }
        tc_commit(drain);
        volatile int never = 0;
        mbar_wait(drain, 0, &never, p.err, kErrWaitConsumer, p.timeout_ns);
      }
    } else {
      // ---------------- MMA issuer ----------------
      reg_dealloc<88>();
      if (lane == 0) {
        const uint32_t q_addr = smem_u32(sq);
        auto qk = [&](int t, int slot) {
          const uint32_t a0 = q_addr + t * C::TILE, b0 = smem_u32(skv + slot * C::TILE);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * C::SUB + (kk & 3) * 32;
            mma_f16_ss(tmem + t * 128, make_sdesc(a0 + off, 16, 1024), make_sdesc(b0 + off, 16, 1024), p.idesc_qk,
                       kk ? 1u : 0u);
          }
        };
        auto pv = [&](int t, int slot, bool first) {
          const uint32_t v0 = smem_u32(skv + slot * C::TILE);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // 128 keys, 16 per MMA; P packs 2 keys per TMEM column
            mma_f16_ts(tmem + 256 + t * D, tmem + t * 128 + kk * 8, make_sdesc(v0 + kk * 2048, C::SUB, 1024),
                       p.idesc_pv, (first && kk == 0) ? 0u : 1u);
        };
        int ring = 0;                 // K/V ring items consumed so far (K_j, V_j of every unit in order)
        int pv_cnt0 = 0, pv_cnt1 = 0;  // PV products issued per Q tile (p_ready phases)
        bool ok = true;
        auto wait_item = [&](int i) {
          return mbar_wait(&kv_full[i % C::SLOTS], (i / C::SLOTS) & 1, abort_flag, p.err, kErrWaitConsumer,
                           p.timeout_ns);
        };
        Unit w;
        for (int k = 0; ok && unit_of<SNAKE>(p, k, w); ++k) {
          auto need = [&](int t, int j) { return j <= (t ? w.last1 : w.last0); };
          const int base = ring;  // K_j is ring item base + 2j, V_j item base + 2j + 1
          auto do_pv = [&](int t, int j, int sv, int &cnt) -> bool {
            if (j == 0 && k > 0) {  // O_t still holds the previous unit until its output has been read
              if (!mbar_wait(&o_free[t], (k - 1) & 1, abort_flag, p.err, kErrWaitSoftmax, p.timeout_ns)) return false;
            }
            if (!mbar_wait(&p_ready[t], cnt & 1, abort_flag, p.err, kErrWaitSoftmax, p.timeout_ns)) return false;
            tc_fence_after();
            pv(t, sv, j == 0);
            tc_commit(&o_ready[t]);
            ++cnt;
            return true;
          };
          if (!(ok = mbar_wait(q_full, k & 1, abort_flag, p.err, kErrWaitConsumer, p.timeout_ns))) break;
          if (!(ok = wait_item(base))) break;
          tc_fence_after();
          if (need(0, 0)) {
            qk(0, base % C::SLOTS);
            tc_commit(&s_ready[0]);
          }
          for (int j = 0; j < w.n_kv; ++j) {
            const int sk = (base + 2 * j) % C::SLOTS, sv = (base + 2 * j + 1) % C::SLOTS;
            if (need(1, j)) {
              qk(1, sk);
              tc_commit(&s_ready[1]);
            }
            // K_j is consumed once both QK products have run; after the last QK, so is Q.
            tc_commit(&kv_empty[sk]);
            if (j + 1 == w.n_kv) tc_commit(q_empty);
            if (!(ok = wait_item(base + 2 * j + 1))) break;
            tc_fence_after();
            if (need(0, j) && !(ok = do_pv(0, j, sv, pv_cnt0))) break;
            if (j + 1 < w.n_kv) {
              if (!(ok = wait_item(base + 2 * (j + 1)))) break;
              tc_fence_after();
              if (need(0, j + 1)) {
                qk(0, (base + 2 * (j + 1)) % C::SLOTS);
                tc_commit(&s_ready[0]);
              }
            }
            if (need(1, j) && !(ok = do_pv(1, j, sv, pv_cnt1))) break;
            tc_commit(&kv_empty[sv]);
          }
          ring = base + 2 * w.n_kv;
        }
        tc_commit(drain);
        volatile int never = 0;
        mbar_wait(drain, 0, &never, p.err, kErrWaitConsumer, p.timeout_ns);
      }
    }
  } else {
    // ---------------- softmax + correction + output (warps 0-7) ----------------
    reg_alloc<208>();
    const int t = warp >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + t * 128;
    const uint32_t o_addr = tmem + lane_base + 256 + t * D;
    int s_cnt = 0;   // S tiles of this Q tile waited for so far (s_ready phases)
    int pv_cnt = 0;  // PV products of this Q tile completed before the current unit (o_ready phases)
    bool ok = true;
    Unit w;
    for (int k = 0; ok && unit_of<SNAKE>(p, k, w); ++k) {
      const int q = w.q0 + 128 * t + row;
      const int last = t ? w.last1 : w.last0;
      const bool tile_valid = t == 0 || w.valid1;
      const int b = w.b, h = w.h;
      float m = -INFINITY, l = 0.0f;
      if (tile_valid) {
        for (int j = 0; j <= last; ++j) {
          if (!(ok = mbar_wait_warp(&s_ready[t], s_cnt & 1, abort_flag, p.err, kErrWaitSoftmax, p.timeout_ns))) break;
          ++s_cnt;
          tc_fence_after();
          const int k0 = j * 128;
          const bool edge = k0 + 127 >= p.Lk || (p.causal && k0 + 127 > w.q0 + 128 * t);
          const bool masked = p.mask_kind != MPC_MASK_NONE && q < p.Lq;
          // The whole 128-key row in registers: four loads in flight, one wait.
          uint32_t r0[32], r1[32], r2[32], r3[32];
          tmem_ld32(s_addr, r0);
          tmem_ld32(s_addr + 32, r1);
          tmem_ld32(s_addr + 64, r2);
          tmem_ld32(s_addr + 96, r3);
          tmem_ld_wait(r0);
          tmem_ld_wait(r1);
          tmem_ld_wait(r2);
          tmem_ld_wait(r3);
          float v[128];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            v[e] = __uint_as_float(r0[e]);
            v[32 + e] = __uint_as_float(r1[e]);
            v[64 + e] = __uint_as_float(r2[e]);
            v[96 + e] = __uint_as_float(r3[e]);
          }
          // Scores stay unscaled (scale > 0 commutes with the max) unless a mask must be added.
          float scl = p.scale_log2;
          if (edge) {
#pragma unroll
            for (int c = 0; c < 128; ++c) {
              const int kc = k0 + c;
              if (kc >= p.Lk || (p.causal && kc > q)) v[c] = -INFINITY;
            }
          }
          if (masked || scl < 0.0f) {
#pragma unroll
            for (int c = 0; c < 128; ++c)
              v[c] = fmaf(v[c], scl, (masked && k0 + c < p.Lk) ? mask_add(p, b, h, q, k0 + c) : 0.0f);
            scl = 1.0f;
          }
          float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int c = 0; c < 128; c += 2) mx[(c >> 1) & 3] = max3f(mx[(c >> 1) & 3], v[c], v[c + 1]);
          const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * scl;
          const float m_new = fmaxf(m, mt);
          const bool grow = m_new > m + 8.0f;  // lazy rescale: P stays below 2^8 otherwise
          if (__any_sync(0xffffffffu, grow)) {
            const float factor = (m == -INFINITY) ? 0.0f : exp2f(m - m_new);
            if (j > 0) {
              if (!(ok = mbar_wait_warp(&o_ready[t], (pv_cnt + j - 1) & 1, abort_flag, p.err, kErrWaitSoftmax,
                                        p.timeout_ns)))
                break;
              tc_fence_after();
#pragma unroll 1
              for (int c = 0; c < D / 32; ++c) {
                uint32_t r[32];
                tmem_ld32(o_addr + c * 32, r);
                tmem_ld_wait(r);
#pragma unroll
                for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * factor);
                tmem_st32(o_addr + c * 32, r);
              }
              tmem_st_wait();
            }
            l *= factor;
            m = m_new;
          }
          const float neg_m = m == -INFINITY ? 0.0f : -m;
          // P = exp2(s·scale - m), packed two keys per TMEM column (key 2e in the low half of column
          // e), over the first 64 S columns (the row is already in registers). The exponentials run
          // two at a time on the f16x2 path of the special-function unit; the argument's f16
          // rounding perturbs P by at most 2^-11·ln2·|x| relative (<= 0.6% for the P < 2^-8 that
          // |x| > 8 gives). The row sum stays f32 (mixed-precision adds of the f16 values).
          float rs[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
          uint32_t w0[32], w1[32];
#pragma unroll
          for (int e = 0; e < 64; ++e) {
            const float2 a = fma2(v[2 * e], v[2 * e + 1], scl, scl, neg_m, neg_m);  // s*scale - m, two at once
            const __half2 x2 = __floats2half2_rn(a.x, a.y);
            const uint32_t e2 = ex2_f16x2(*reinterpret_cast<const uint32_t *>(&x2));
            uint32_t packed = e2;
            if (BF) {
              // bf16 P: the row sum adds the rounded values P.V uses, so that O / l stays a convex
              // combination of V rows (the weights' common rounding cancels in the quotient).
              const float2 pf = __half22float2(*reinterpret_cast<const __half2 *>(&e2));
              __nv_bfloat162 v2 = __floats2bfloat162_rn(pf.x, pf.y);
              packed = *reinterpret_cast<uint32_t *>(&v2);
              rs[e & 7] += __uint_as_float(packed << 16) + __uint_as_float(packed & 0xFFFF0000u);
            } else {
              rs[e & 7] = add_f16x2_to_f32(rs[e & 7], e2);
            }
            if (e < 32)
              w0[e] = packed;
            else
              w1[e - 32] = packed;
          }
          tmem_st32(s_addr, w0);
          tmem_st32(s_addr + 32, w1);
          l += ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_ready[t]);
        }
        if (!ok) break;
        // ---- output: O / l, rows below Lq ----
        if (!(ok = mbar_wait_warp(&o_ready[t], (pv_cnt + last) & 1, abort_flag, p.err, kErrWaitSoftmax,
                                  p.timeout_ns)))
          break;
        pv_cnt += last + 1;
        tc_fence_after();
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
        const size_t orow = (size_t)w.b * p.os[0] + (size_t)w.h * p.os[1] + (size_t)q * p.os[2];
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(o_addr + c * 32, r);
          tmem_ld_wait(r);
          if (c + 1 == D / 32) {  // O_t is in registers: the next unit's first PV may overwrite it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_free[t]);
          }
          if (q < p.Lq) {
            uint32_t ow[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const float a = __uint_as_float(r[2 * e]) * inv, bb = __uint_as_float(r[2 * e + 1]) * inv;
              if (BF) {
                __nv_bfloat162 v2 = __floats2bfloat162_rn(a, bb);
                ow[e] = *reinterpret_cast<uint32_t *>(&v2);
              } else {
                __half2 v2 = __floats2half2_rn(a, bb);
                ow[e] = *reinterpret_cast<uint32_t *>(&v2);
              }
            }
            uint4 *dst = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.out) + orow + c * 32);
#pragma unroll
            for (int e = 0; e < 4; ++e) dst[e] = make_uint4(ow[4 * e], ow[4 * e + 1], ow[4 * e + 2], ow[4 * e + 3]);
          }
        }
        if (p.lse && q < p.Lq)
          p.lse[(size_t)w.bh * p.Lq + q] = l > 0.0f ? (m * 0.6931471805599453f + logf(l)) : -INFINITY;
      } else {
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_free[t]);  // keep o_free's phases in step with the units
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------------------------
// Generic CUDA-core path: one warp per query row, keys in chunks of 32 (lane = key), f32 math.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float ld(const void *p, int dt, size_t i) {
  if (dt == MPC_F32) return static_cast<const float *>(p)[i];
  if (dt == MPC_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
  return __half2float(static_cast<const __half *>(p)[i]);
}
__device__ __forceinline__ void st(void *p, int dt, size_t i, float v) {
  if (dt == MPC_F32)
    static_cast<float *>(p)[i] = v;
  else if (dt == MPC_BF16)
    static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
  else
    static_cast<__half *>(p)[i] = __float2half_rn(v);
}

struct GenericParams {
  int B, H, Hk, Lq, Lk, D, Dv, rep, causal, dtype, mask_kind;
  float scale;
  const void *q, *k, *v, *mask;
  long long ms[4];
  long long qs[3], ks[3], vs[3], os[3];  // element strides of (batch, head, row)
  void *out;
  float *lse;
};

__global__ void attn_generic_kernel(const GenericParams p) {
  __shared__ float qs[8][256];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row_id = (long long)blockIdx.x * 8 + w;  // over B*H*Lq
  const long long rows = (long long)p.B * p.H * p.Lq;
  if (row_id >= rows) return;
  const int q = (int)(row_id % p.Lq);
  const int bh = (int)(row_id / p.Lq);
  const int b = bh / p.H, h = bh % p.H;
  const int kvh = h / p.rep;
  const size_t qrow = (size_t)b * p.qs[0] + (size_t)h * p.qs[1] + (size_t)q * p.qs[2];
  const size_t kbase = (size_t)b * p.ks[0] + (size_t)kvh * p.ks[1];
  const size_t vbase = (size_t)b * p.vs[0] + (size_t)kvh * p.vs[1];
  for (int d = lane; d < p.D; d += 32) qs[w][d] = ld(p.q, p.dtype, qrow + d);
  __syncwarp();
  float m = -INFINITY, l = 0.0f;
  float o[8];  // dims lane, lane+32, ..., Dv <= 256
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = 0.0f;
  const int k_end = p.causal ? min(p.Lk, q + 1) : p.Lk;
  for (int k0 = 0; k0 < k_end; k0 += 32) {
    const int k = k0 + lane;
    float s = -INFINITY;
    if (k < k_end) {
      float acc = 0.0f;
      const size_t kb = kbase + (size_t)k * p.ks[2];
      for (int d = 0; d < p.D; ++d) acc = fmaf(qs[w][d], ld(p.k, p.dtype, kb + d), acc);
      s = acc * p.scale;
      if (p.mask_kind != MPC_MASK_NONE) {
        const long long off = b * p.ms[0] + h * p.ms[1] + q * p.ms[2] + k * p.ms[3];
        if (p.mask_kind == MPC_MASK_BOOL)
          s = static_cast<const uint8_t *>(p.mask)[off] ? s : -INFINITY;
        else
          s += static_cast<const float *>(p.mask)[off];
      }
    }
    float mt = s;
#pragma unroll
    for (int o2 = 16; o2; o2 >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o2));
    const float m_new = fmaxf(m, mt);
    if (m_new == -INFINITY) continue;  // nothing visible yet
    const float factor = m == -INFINITY ? 0.0f : expf(m - m_new);
    const float pk = s == -INFINITY ? 0.0f : expf(s - m_new);
    float ps = pk;
#pragma unroll
    for (int o2 = 16; o2; o2 >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o2);
    l = l * factor + ps;
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] *= factor;
    const int nk = min(32, k_end - k0);
    for (int jj = 0; jj < nk; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, pk, jj);
      if (pj == 0.0f) continue;  // masked keys contribute nothing (even a non-finite V row)
      const size_t vb = vbase + (size_t)(k0 + jj) * p.vs[2];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int d = lane + 32 * i;
        if (d < p.Dv) o[i] = fmaf(pj, ld(p.v, p.dtype, vb + d), o[i]);
      }
    }
    m = m_new;
  }
  const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = lane + 32 * i;
    if (d < p.Dv) st(p.out, p.dtype, (size_t)b * p.os[0] + (size_t)h * p.os[1] + (size_t)q * p.os[2] + d, o[i] * inv);
  }
  if (p.lse && lane == 0) p.lse[row_id] = l > 0.0f ? m + logf(l) : -INFINITY;
}

// Whether the snake order (unit_of<true>) spreads a causal launch's work more evenly than the pairs: the
// largest per-CTA sum of unit costs (KV tiles of both Q tiles, plus one for the unit's output) under
// each order, the snake kept when it is at least 3% lower. Beyond 2^16 units the pairs' rounding
// loss is below half a percent and the pairs stay.
static bool prefer_snake(const Params &p, long long grid_pairs, long long grid_snake) {
  if (p.n_units > (1 << 16) || grid_pairs <= 0 || grid_snake <= 0) return false;
  const int qbn = p.q_blocks;
  const long long bhn = p.n_units / qbn;
  std::vector<long long> cost(qbn);
  for (int qb = 0; qb < qbn; ++qb) {
    const int q0 = qb * 256;
    const bool valid1 = q0 + 128 < p.Lq;
    cost[qb] = (last_kv(p, q0) + 1) + (valid1 ? last_kv(p, q0 + 128) + 1 : 0) + 1;
  }
  std::vector<long long> a(grid_pairs, 0), b(grid_snake, 0);
  for (long long u = 0; u < p.n_units; ++u) {
    const int r = (int)(u % qbn);
    a[(u / 2) % grid_pairs] += cost[(r & 1) ? (r >> 1) : qbn - 1 - (r >> 1)];
    const long long k = u / grid_snake, i = u % grid_snake;
    b[(k & 1) ? grid_snake - 1 - i : i] += cost[qbn - 1 - (int)(u / bhn)];
  }
  const long long ma = *std::max_element(a.begin(), a.end()), mb = *std::max_element(b.begin(), b.end());
  return mb * 100 < ma * 97;
}

template <int D, bool BF, bool SNAKE, bool DUAL>
int launch_order(mpc_device *dev, const Maps &maps, const Params &p, long long grid, cudaStream_t st) {
  using C = Cfg<D>;
  static bool configured[64] = {};
  const int ord = dev->ordinal & 63;
  if (!configured[ord]) {
    MPC_CUDA(dev, cudaFuncSetAttribute(attn_kernel<D, BF, SNAKE, DUAL>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    cudaFuncAttributes fa;
    MPC_CUDA(dev, cudaFuncGetAttributes(&fa, attn_kernel<D, BF, SNAKE, DUAL>));
    // The register split inside the kernel is sized for a 168-register launch; refuse anything else
    // rather than launch a split whose increase could never be granted.
    if (fa.numRegs != 168)
      return fail(MPC_ERR_UNSUPPORTED, "attn_kernel built with %d registers per thread (expected 168)", fa.numRegs);
    configured[ord] = true;
  }
  attn_kernel<D, BF, SNAKE, DUAL><<<(unsigned)grid, C::THREADS, C::SMEM, st>>>(maps, p);
  dev->launches++;
  return check_launch(dev, "attn_kernel");
}

// Persistent: one CTA per SM (at most), each taking units until none is left. The unit order and
// the MMA issuers are separate instantiations, so that no kernel carries a branch for the others.
// Measured (causal, A/B on one box each time): [8,16,1024,128] bf16 383-422 TFLOP/s with one
// issuer per tile against 364-369 with one stream; [16,16,512,128] f16 318 against 292-313;
// [32,12,1024,64] f16 306-314 against 293-301; [32,12,1536,64] bf16 307-314 against 293-302; but
// [16,32,1280,128] f16 625 against 664, [16,32,1536,128] f16 658 against 704, [16,32,2048,128] f16
// 707 against 814, [16,12,2048,64] bf16 361 against 382, [8,12,4096,64] bf16 394 against 443, and
// non-causal rows 756-774 against 873-1009, so those keep the one stream.
template <int D, bool BF>
int launch_tc(mpc_device *dev, const Maps &maps, const Params &p, cudaStream_t st) {
  const long long sms = dev->prop.multiProcessorCount;
  const long long pairs = ((long long)p.n_units + 1) / 2;
  const long long grid = pairs < sms ? pairs : sms;
  const long long grid_snake = p.n_units < sms ? p.n_units : sms;
  if (!p.causal) return launch_order<D, BF, false, false>(dev, maps, p, grid, st);
  const bool snake = prefer_snake(p, grid, grid_snake);
  if (p.Lk <= (D == 64 ? 1536 : 1024))
    return snake ? launch_order<D, BF, true, true>(dev, maps, p, grid_snake, st)
                 : launch_order<D, BF, false, true>(dev, maps, p, grid, st);
  return snake ? launch_order<D, BF, true, false>(dev, maps, p, grid_snake, st)
               : launch_order<D, BF, false, false>(dev, maps, p, grid, st);
}

}  // namespace attn

namespace attn {
// A 4-D map over one of Q / K / V: axes (head-dim, then head / row / batch sorted by stride so the
// map's strides increase); the box is 64 columns x 128 rows. *pos receives each logical axis's map
// position (head bits 0-1, row bits 2-3, batch bits 4-5).
static int rows_map(CUtensorMap *map, CUtensorMapDataType dt, const void *base, int64_t d, int64_t heads,
                    int64_t rows, int64_t batch, const int64_t st[3], int *pos) {
  struct Ax {
    int64_t extent, stride;
    int logical;  // 0 head, 1 row, 2 batch
  } ax[3] = {{heads, st[1], 0}, {rows, st[2], 1}, {batch, st[0], 2}};
  int64_t top = d;
  for (auto &a : ax) top = std::max(top, a.stride * a.extent);
  for (auto &a : ax)
    if (a.extent == 1) a.stride = top;  // a unit axis never moves: any valid stride
  std::sort(ax, ax + 3, [](const Ax &x, const Ax &y) { return x.stride < y.stride; });
  uint64_t dims[4] = {(uint64_t)d, 0, 0, 0}, strides[3];
  uint32_t box[4] = {64, 1, 1, 1};
  *pos = 0;
  for (int i = 0; i < 3; ++i) {
    dims[i + 1] = (uint64_t)ax[i].extent;
    strides[i] = (uint64_t)ax[i].stride * 2;
    if (ax[i].logical == 1) box[i + 1] = 128;
    *pos |= (i + 1) << (2 * ax[i].logical);
  }
  return make_map_4d(map, dt, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}
}  // namespace attn

int sdpa_run(mpc_device *dev, const mpc_sdpa_desc *d, const void *Q, const void *K, const void *V, const void *mask,
             void *O, float *LSE, const mpc_sdpa_layout *layout, cudaStream_t st) {
  using namespace attn;
  if (d->b < 0 || d->h <= 0 || d->hk <= 0 || d->lq < 0 || d->lk < 0 || d->d <= 0 || d->dv <= 0)
    return fail(MPC_ERR_INVALID, "mpc_sdpa: bad extents b=%lld h=%lld hk=%lld lq=%lld lk=%lld d=%lld dv=%lld",
                (long long)d->b, (long long)d->h, (long long)d->hk, (long long)d->lq, (long long)d->lk,
                (long long)d->d, (long long)d->dv);
  if (d->h % d->hk) return fail(MPC_ERR_INVALID, "mpc_sdpa: H=%lld is not a multiple of Hk=%lld", (long long)d->h,
                                (long long)d->hk);
  if (d->dtype != MPC_F32 && d->dtype != MPC_F16 && d->dtype != MPC_BF16)
    return fail(MPC_ERR_INVALID, "mpc_sdpa: dtype %d", d->dtype);
  if (d->mask_kind < MPC_MASK_NONE || d->mask_kind > MPC_MASK_ADD || (d->mask_kind && !mask))
    return fail(MPC_ERR_INVALID, "mpc_sdpa: mask_kind %d with mask %p", d->mask_kind, mask);
  if (d->b == 0 || d->lq == 0) return MPC_OK;
  if (!Q || !K || !V || !O) return fail(MPC_ERR_INVALID, "mpc_sdpa: null operand");
  if (d->b * d->h > (1 << 30) || d->lq > (1 << 30) || d->lk > (1 << 30))
    return fail(MPC_ERR_UNSUPPORTED, "mpc_sdpa: extents above 2^30");
  mpc_sdpa_layout lay;
  if (layout) {
    lay = *layout;
    for (const int64_t *v : {lay.q, lay.k, lay.v, lay.o})
      for (int i = 0; i < 3; ++i)
        if (v[i] < 0) return fail(MPC_ERR_INVALID, "mpc_sdpa_strided: negative stride");
  } else {  // contiguous [B, H, L, D]
    const int64_t q[3] = {d->h * d->lq * d->d, d->lq * d->d, d->d};
    const int64_t k[3] = {d->hk * d->lk * d->d, d->lk * d->d, d->d};
    const int64_t v[3] = {d->hk * d->lk * d->dv, d->lk * d->dv, d->dv};
    const int64_t o[3] = {d->h * d->lq * d->dv, d->lq * d->dv, d->dv};
    for (int i = 0; i < 3; ++i) lay.q[i] = q[i], lay.k[i] = k[i], lay.v[i] = v[i], lay.o[i] = o[i];
  }
  bool strides16 = true;
  for (const int64_t *v : {lay.q, lay.k, lay.v, lay.o})
    for (int i = 0; i < 3; ++i) strides16 = strides16 && (v[i] * 2) % 16 == 0;
  const bool aligned = !((uintptr_t)Q & 15) && !((uintptr_t)K & 15) && !((uintptr_t)V & 15) && !((uintptr_t)O & 15);
  const bool tc = d->dtype != MPC_F32 && d->d == d->dv && (d->d == 64 || d->d == 128) && aligned && strides16 &&
                  d->lk > 0;
  if (!tc) {
    if (d->d > 256 || d->dv > 256) return fail(MPC_ERR_UNSUPPORTED, "mpc_sdpa: head dim above 256");
    GenericParams g{};
    g.B = (int)d->b, g.H = (int)d->h, g.Hk = (int)d->hk, g.Lq = (int)d->lq, g.Lk = (int)d->lk, g.D = (int)d->d;
    g.Dv = (int)d->dv, g.rep = (int)(d->h / d->hk), g.causal = d->causal ? 1 : 0, g.dtype = d->dtype;
    g.mask_kind = d->mask_kind, g.scale = d->scale, g.q = Q, g.k = K, g.v = V, g.mask = mask, g.out = O, g.lse = LSE;
    for (int i = 0; i < 4; ++i) g.ms[i] = d->mask_strides[i];
    for (int i = 0; i < 3; ++i) g.qs[i] = lay.q[i], g.ks[i] = lay.k[i], g.vs[i] = lay.v[i], g.os[i] = lay.o[i];
    const long long rows = d->b * d->h * d->lq;
    attn_generic_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(g);
    dev->launches++;
    return check_launch(dev, "attn_generic_kernel");
  }
  Params p{};
  p.B = (int)d->b, p.H = (int)d->h, p.Hk = (int)d->hk, p.Lq = (int)d->lq, p.Lk = (int)d->lk, p.D = (int)d->d;
  p.rep = p.H / p.Hk;
  p.q_blocks = (p.Lq + 255) / 256;
  const long long units = (long long)p.q_blocks * p.B * p.H;
  if (2 * units + 2 * dev->prop.multiProcessorCount >= (1ll << 31))
    return fail(MPC_ERR_UNSUPPORTED, "mpc_sdpa: %lld units of 256 query rows (at most 2^30)", units);
  p.n_units = (int)units;
  p.causal = d->causal ? 1 : 0;
  p.scale_log2 = d->scale * 1.4426950408889634f;
  p.mask_kind = d->mask_kind;
  p.mask = mask;
  for (int i = 0; i < 4; ++i) p.ms[i] = d->mask_strides[i];
  p.out = O;
  for (int i = 0; i < 3; ++i) p.os[i] = lay.o[i];
  p.lse = LSE;
  p.dtype = d->dtype;
  const uint32_t fmt = d->dtype == MPC_BF16 ? kFmtBF16 : kFmtF16;
  p.idesc_qk = make_idesc(fmt, false, 128, 128);
  p.idesc_pv = make_idesc(fmt, true, 128, p.D);
  p.err = dev->d_err;
  p.timeout_ns = dev->timeout_ns;
  Maps maps;
  memset(&maps, 0, sizeof(maps));
  const CUtensorMapDataType dt = d->dtype == MPC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  int rc, kpos = 0, vpos = 0;
  if ((rc = rows_map(&maps.q, dt, Q, p.D, p.H, p.Lq, p.B, lay.q, &p.q_pos)) ||
      (rc = rows_map(&maps.k, dt, K, p.D, p.Hk, p.Lk, p.B, lay.k, &kpos)) ||
      (rc = rows_map(&maps.v, dt, V, p.D, p.Hk, p.Lk, p.B, lay.v, &vpos)))
    return rc;
  p.k_pos = kpos;
  p.v_pos = vpos;
  const bool bf = p.dtype == MPC_BF16;
  if (p.D == 128) return bf ? launch_tc<128, true>(dev, maps, p, st) : launch_tc<128, false>(dev, maps, p, st);
  return bf ? launch_tc<64, true>(dev, maps, p, st) : launch_tc<64, false>(dev, maps, p, st);
}

}  // namespace mpc
