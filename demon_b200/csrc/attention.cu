// attention.cu -- bidirectional grouped-query attention of the DiT on sm_100a:
//   O = softmax(Q K^T * scale, keys restricted to |i - j| <= window when a window is given) V
// for head_dim 128, bf16 Q / K / V / O, fp32 scores and softmax.
//
// Stands in for the attention core of AceStepAttention.forward
// (acestep/models/modeling_acestep_v15_turbo.py:358-372: the attention interface called with
// sliding_window for the "sliding_attention" layers and None for the others and for cross
// attention), whose bidirectional band is |i - j| <= sliding_window (same file, 110-112) --
// scaled_dot_product_attention over the GQA-shared K / V heads.
//
// Work unit: one (sequence, kv head, pair of q heads of that kv head, 128-query block).  Both
// q heads read the same K / V tiles, so each 128-key K / V tile is loaded into shared memory
// once per unit and used by four MMAs (S = Q K^T and O += P V for each head).  Persistent
// CTAs (one per SM) walk the units in a static round-robin; a band unit visits its diagonal
// key tile first (rows then start from a running maximum over 128 keys).
//
// Warp roles (512 threads, four warpgroups; setmaxnreg moves registers from the epilogue and
// issuing warpgroups to the softmax warpgroups):
//   warpgroup 0 / 1  softmax of q head 0 / 1 of the unit, one query row per thread,
//   warpgroup 2      epilogue: O_h / rowsum -> bf16 -> swizzled shared memory -> TMA store,
//   warp 12          TMA loads: Q tiles into a 3-slot ring, K / V tiles into a 3-slot ring,
//   warp 13          MMA issue (one thread) and tensor-memory allocation.
// Tensor memory (512 columns): S_h at 128 h, O_h at 256 + 128 h (fp32, row = lane); P_h, the
// bf16 probabilities, overwrite the upper half of S_h (columns 128 h + 64 ..) and feed the
// P V MMA straight from tensor memory.  The MMAs of one thread run in issue order, which is
// what lets the next S_h = Q K^T overwrite P_h: it is issued after the P V that reads it.
//
// MMA order, the units of a CTA forming one stream of key tiles (i = tile of the unit):
//   QK0(i) PV1(i-1) QK1(i) PV0(i)
// with PV1 of a unit's last tile issued after the next unit's QK0(0), so the softmax of
// head 0 runs on into the next unit while head 1 finishes.  Each PV is issued in two halves
// of 64 keys: the softmax publishes the probabilities of keys 0-63 first, and their product
// runs while it computes those of keys 64-127.  The commit that signals S_h(i) also covers
// PV_h(i-1): when a softmax warp sees S_h(i), no MMA touches O_h until it publishes P_h(i),
// so it may rescale O_h in place.
//
// Softmax (per row, log2 domain): t = s * scale * log2(e).  The running offset m is only
// raised when a tile's row maximum exceeds it by more than 8 (then O_h and the row sum are
// rescaled by 2^(m_old - m_new)); otherwise the stale offset stays, so p = 2^(t - m) <= 256.
// Numerator and denominator use the same offset, so the result is the exact softmax up to
// rounding (the lazy rescaling of FlashAttention-4, Dao et al. 2025).
//
// Epilogue: after a unit's last P V of head h, the epilogue warps read O_h from tensor memory
// (and hand its columns back to the MMA warp), scale each row by 1 / rowsum (handed over by
// the softmax warps through shared memory) and store the bf16 rows with per-warp TMA stores
// (rows past the sequence end are clipped by the tensor map).
//
// Every wait is a bounded mbarrier wait; on expiry the kernel records DEMON_DEV_TIMEOUT in
// the status word, every role leaves its loop, outstanding copies and MMAs are waited for
// (bounded) and the tensor memory is freed.
#include <algorithm>
#include <cstring>

#include "demon_common.cuh"
#include "demon_host.h"

namespace demon {
namespace attn {

constexpr int kD = 128;                 // head dim
constexpr int kBlk = 128;               // queries per block, keys per tile
constexpr int kBox = 128 * 128;         // one 64-column x 128-row bf16 box (16 KB)
constexpr int kTile = 2 * kBox;         // one 128 x 128 bf16 tile (two boxes, 32 KB)
constexpr int kSlots = 3;                    // K / V ring slots
constexpr int kQSlots = 3;                   // Q ring slots (one 128 x 128 tile of one head each)
constexpr int kWarpStg = 2 * 32 * 128;       // one epilogue warp's 32-row O staging (two 4 KB boxes)
constexpr int kThreads = 512;           // four warpgroups

// Registers per thread after the split (setmaxnreg): the launch gives 512 x 128; the two
// softmax warpgroups take 176, the epilogue warpgroup 56, the TMA / MMA warpgroup 104:
// 256 * 176 + 128 * 56 + 128 * 104 = 63,536 <= 512 * 128.  No role spills at these counts;
// the issue warpgroup (descriptors and ring phases of both loops) is the one that spilled at
// 64 (176 bytes), which delayed MMA issue: band attention 394 -> 383 us, global 563 -> 556 us.
constexpr int kLaunchRegs = 128, kSoftmaxRegs = 176, kEpilogueRegs = 56, kIssueRegs = 104;
static_assert(256 * kSoftmaxRegs + 128 * kEpilogueRegs + 128 * kIssueRegs <= kThreads * kLaunchRegs,
              "register split exceeds the launch's registers (setmaxnreg.inc would wait for good)");

constexpr int offQ = 0;                                 // Q ring (96 KB)
constexpr int offKV = offQ + kQSlots * kTile;           // K / V ring (96 KB)
constexpr int offStg = offKV + kSlots * kTile;          // 4 epilogue warps x 8 KB
constexpr int offL = offStg + 4 * kWarpStg;             // row sums: [2 heads][128 rows] fp32
constexpr int offBar = offL + 2 * 128 * 4;              // mbarriers
constexpr int kNumBars = 2 * kQSlots + 2 * kSlots + 2 * 7 + 1;
constexpr int offMisc = offBar + kNumBars * 8;          // tmem holder, abort flag
constexpr int kSmemUsed = offMisc + 16;
constexpr int kSmem = kSmemUsed + 1024;                 // + alignment slack
static_assert(kSmem <= 232448, "attention shared memory exceeds the sm_100 per-block limit");

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColP = 64, kColO = 256;  // S_h at 128 h, P_h at 128 h + 64, O_h at 256 + 128 h
constexpr float kRescaleLog2 = 8.0f;                    // lazy rescale threshold (log2 units)

// Division by a divisor fixed for the launch (Granlund and Montgomery, "Division by invariant
// integers using multiplication", PLDI 1994, theorem 4.2): with l = ceil(log2 d), s = 31 + l and
// m = ceil(2^s / d), floor(n / d) = (n * m) >> s for every 0 <= n < 2^31 (m * d - 2^s < d <=
// 2^(s - 31)), and m < 2^32.  The work-unit decode below runs at every unit boundary in each
// role, the MMA thread's between one unit's last P V and the next unit's first Q K^T; a 64-bit
// division there is a long dependent instruction sequence.
struct FastDiv {
  uint32_t d, m, s;
};
__host__ __device__ inline FastDiv make_fastdiv(uint32_t d) {
  uint32_t l = 0;
  while (l < 32 && (1ull << l) < d) ++l;
  const uint32_t s = 31 + l;
  return FastDiv{d, (uint32_t)(((1ull << s) + d - 1) / d), s};
}
__device__ __forceinline__ uint32_t fast_div(uint32_t n, const FastDiv& f) {
  return (uint32_t)(((uint64_t)n * f.m) >> f.s);
}

struct Params {
  int B, S, L, Hk, G, window;  // window < 0: no band
  int n_qblk, n_kblk, pairs;   // blocks of 128 queries, tiles of 128 keys, q-head pairs per kv head
  FastDiv div_qblk, div_pairs, div_hk;
  float scale_log2;            // softmax scale * log2(e)
  int64_t units;               // < 2^31 (checked on the host)
  unsigned int* status;
};

struct Unit {
  int b, hk, h0, qb, kt0, nt;  // sequence, kv head, first q head, query block, first key tile, tiles
  int ktd;                     // key tile visited first (the band's diagonal tile; kt0 without a band)
};

// Key tile of step i of a unit: the diagonal tile first, then the others in order.  With a
// band, rows whose first tile held only a few keys of their range would start from a poor
// running maximum, and the next tile's would exceed it by more than 2^8 (an O rescale).
__device__ __forceinline__ int key_tile(const Unit& w, int i) {
  if (i == 0) return w.ktd;
  const int k = w.kt0 + i - 1;
  return k < w.ktd ? k : k + 1;
}

__device__ __forceinline__ Unit decode(const Params& p, int64_t u) {
  Unit w;
  const uint32_t n = (uint32_t)u;  // u < units < 2^31
  const uint32_t r1 = fast_div(n, p.div_qblk);
  w.qb = (int)(n - r1 * p.div_qblk.d);
  const uint32_t r2 = fast_div(r1, p.div_pairs);
  const int pair = (int)(r1 - r2 * p.div_pairs.d);
  const uint32_t r3 = fast_div(r2, p.div_hk);
  w.hk = (int)(r2 - r3 * p.div_hk.d);
  w.b = (int)r3;
  w.h0 = w.hk * p.G + 2 * pair;
  const int q0 = w.qb * kBlk;
  if (p.window >= 0) {
    const int qlast = min(q0 + kBlk - 1, p.S - 1);
    const int klo = max(0, q0 - p.window);
    const int khi = min(p.L - 1, qlast + p.window);
    w.kt0 = klo / kBlk;
    w.nt = khi / kBlk - w.kt0 + 1;
    w.ktd = min(max(q0 / kBlk, w.kt0), w.kt0 + w.nt - 1);
  } else {
    w.kt0 = 0;
    w.nt = p.n_kblk;
    w.ktd = 0;
  }
  return w;
}

// K-major, 128-byte-swizzled operand (Q or K): k-step kk (16 elements) of a 128 x 128 tile.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile, int kk) {
  return smem_desc(tile + (uint32_t)(kk >> 2) * kBox + (uint32_t)(kk & 3) * 32, 16, 1024, 2);
}
// MN-major, 128-byte-swizzled B operand (V, d contiguous): keys 16 kk .. 16 kk + 15.  Rows
// of 8 keys are 1024 B apart (stride byte offset), the two 64-column boxes 16 KB apart
// (leading byte offset).
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile, int kk) {
  return smem_desc(tile + (uint32_t)kk * 2048, kBox, 1024, 2);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// A warp-uniform bounded wait: every lane waits, and the warp proceeds only if all did.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, uint64_t t0,
                                          unsigned int* status, unsigned int where) {
  const bool ok = mbar_wait(bar, parity, abort, t0, status, where);
  return __all_sync(0xffffffffu, ok && *abort == 0);
}

template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                     const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + offBar);
  // Q tiles go through their own ring in the order (unit 0, head 0), (unit 0, head 1),
  // (unit 1, head 0), ...: Q tile 2 it + h of a CTA sits in slot (2 it + h) % 3, so the next
  // unit's Q loads while the current unit still runs.
  uint64_t* q_full = bars + 0;                         // [3] TMA -> MMA: Q tile loaded
  uint64_t* q_empty = bars + kQSlots;                  // [3] MMA -> TMA: its last S computed
  uint64_t* kv_full = bars + 2 * kQSlots;
  uint64_t* kv_empty = bars + 2 * kQSlots + kSlots;
  uint64_t* s_full = bars + 2 * kQSlots + 2 * kSlots;  // [2] MMA -> softmax: S_h computed
  uint64_t* pa_full = s_full + 2;            // [2] softmax -> MMA: P_h of keys 0-63 in tensor memory
  uint64_t* pb_full = s_full + 4;            // [2] softmax -> MMA: P_h of keys 64-127
  uint64_t* o_full = s_full + 6;             // [2] MMA -> epilogue: the unit's last P V done
  uint64_t* o_empty = s_full + 8;            // [2] epilogue -> MMA: O_h read out
  uint64_t* l_full = s_full + 10;            // [2] softmax -> epilogue: row sums written
  uint64_t* l_empty = s_full + 12;           // [2] epilogue -> softmax: row sums read
  uint64_t* mma_done = s_full + 14;
  const uint32_t lbuf = sbase + offL;        // [2][128] fp32
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + offMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + offMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t t0 = globaltimer();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kQSlots; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&s_full[h], 1);
      mbar_init(&pa_full[h], 4);  // one arrive per softmax warp
      mbar_init(&pb_full[h], 4);
      mbar_init(&o_full[h], 1);
      mbar_init(&o_empty[h], 4);  // one arrive per epilogue warp
      mbar_init(&l_full[h], 4);   // one arrive per softmax warp
      mbar_init(&l_empty[h], 4);  // one arrive per epilogue warp
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 12 && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmO);
  }
  if (warp == 13) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int64_t stride = gridDim.x;
  const int wg = warp >> 2;

  if (wg == 3) {
    setmaxnreg_dec<kIssueRegs>();
    if (warp == 12) {
      // ---------------------------------------------------------- TMA producer
      if (elect_one()) {
        uint32_t g = 0, it = 0, nq = 0;  // K / V tiles issued, units started, Q tiles issued
        bool ok = true;
        auto load_q = [&](const Unit& w, int h) {
          const int s = (int)(nq % kQSlots);
          if (!(ok = mbar_wait(&q_empty[s], ((nq / kQSlots) & 1u) ^ 1u, abort_flag, t0, p.status, 21))) return false;
          mbar_arrive_expect_tx(&q_full[s], kTile);
          for (int half = 0; half < 2; ++half)
            tma_load_3d(sbase + offQ + s * kTile + half * kBox, &tmQ, &q_full[s], (w.h0 + h) * kD + half * 64,
                        w.qb * kBlk, w.b);
          ++nq;
          return true;
        };
        // order per unit: Q of head 0, K / V of the first key tile, Q of head 1, the other tiles
        // (the MMA issues the unit's first S_0 before the previous unit's last P_1 V)
        for (int64_t u = blockIdx.x; ok && u < p.units; u += stride, ++it) {
          const Unit w = decode(p, u);
          if (!load_q(w, 0)) break;
          for (int i = 0; ok && i < w.nt; ++i) {
            const int k0 = key_tile(w, i) * kBlk;
            for (int kv = 0; kv < 2; ++kv, ++g) {
              const int s = (int)(g % kSlots);
              if (!(ok = mbar_wait(&kv_empty[s], ((g / kSlots) & 1u) ^ 1u, abort_flag, t0, p.status, 22))) break;
              mbar_arrive_expect_tx(&kv_full[s], kTile);
              const CUtensorMap* m = kv ? &tmV : &tmK;
              for (int half = 0; half < 2; ++half)
                tma_load_3d(sbase + offKV + s * kTile + half * kBox, m, &kv_full[s], w.hk * kD + half * 64, k0,
                            w.b);
            }
            if (ok && i == 0 && !load_q(w, 1)) break;
          }
        }
        // drain: no copy may still be in flight when the CTA leaves (immediate on the normal path)
        volatile int never = 0;
        for (uint32_t i = g > (uint32_t)kSlots ? g - kSlots : 0; i < g; ++i)
          mbar_wait(&kv_full[i % kSlots], (i / kSlots) & 1u, &never, globaltimer(), p.status, 23);
        for (uint32_t i = nq > (uint32_t)kQSlots ? nq - kQSlots : 0; i < nq; ++i)
          mbar_wait(&q_full[i % kQSlots], (i / kQSlots) & 1u, &never, globaltimer(), p.status, 24);
      }
      __syncwarp();
    } else if (warp == 13) {
      // ---------------------------------------------------------- MMA issuer
      if (elect_one()) {
        const uint32_t idesc_qk = idesc_bf16(kBlk, kBlk);
        const uint32_t idesc_pv = idesc_bf16(kBlk, kD) | (1u << 16);  // B (V) MN-major
        uint32_t g = 0, it = 0, tiles = 0;  // K / V tiles consumed, units, key tiles (all units)
        bool ok = true;
        auto qk = [&](int h, uint32_t kslot) {
          const uint32_t qa = sbase + offQ + ((2 * it + h) % kQSlots) * kTile, kb = sbase + offKV + kslot * kTile;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_bf16(tmem + kColS + 128 * h, kmajor_desc(qa, kk), kmajor_desc(kb, kk), idesc_qk, kk > 0);
          tc_commit(&s_full[h]);
        };
        // O_h += P_h V over keys 64 half .. 64 half + 63 (acc = 0: the unit's first product)
        auto pv = [&](int h, uint32_t vslot, int half, bool acc) {
          const uint32_t vb = sbase + offKV + vslot * kTile;
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) {
            const int kk = 4 * half + k4;
            mma_bf16_ts(tmem + kColO + 128 * h, tmem + kColS + 128 * h + kColP + 8 * kk, mnmajor_desc(vb, kk),
                        idesc_pv, (acc || kk > 0) ? 1u : 0u);
          }
        };
        auto wait_kv = [&](uint32_t gi) {
          ok = mbar_wait(&kv_full[gi % kSlots], (gi / kSlots) & 1u, abort_flag, t0, p.status, 31);
          if (ok) tc_fence_after();
          return ok;
        };
        auto wait_p = [&](uint64_t* bar, int h, uint32_t t) {
          ok = mbar_wait(&bar[h], t & 1u, abort_flag, t0, p.status, 32 + h);
          if (ok) tc_fence_after();
          return ok;
        };
        // both halves of P_h(t) into O_h: the first as soon as it is published
        auto pv_tile = [&](int h, uint32_t vslot, uint32_t t, bool acc) {
          if (!wait_p(pa_full, h, t)) return false;
          pv(h, vslot, 0, acc);
          if (!wait_p(pb_full, h, t)) return false;
          pv(h, vslot, 1, true);
          return true;
        };
        auto wait_oe = [&](int h) {
          ok = mbar_wait(&o_empty[h], (it & 1u) ^ 1u, abort_flag, t0, p.status, 34 + h);
          if (ok) tc_fence_after();
          return ok;
        };
        auto wait_q = [&](int h) {
          const uint32_t qi = 2 * it + h;
          ok = mbar_wait(&q_full[qi % kQSlots], (qi / kQSlots) & 1u, abort_flag, t0, p.status, 30);
          if (ok) tc_fence_after();
          return ok;
        };
        auto free_q = [&](int h) { tc_commit(&q_empty[(2 * it + h) % kQSlots]); };
        // The units form one stream of key tiles: the last P_1 V of a unit is issued after the
        // next unit's first S_0 = Q K^T, as inside a unit, so head 0's softmax goes on without
        // waiting for the unit boundary.
        bool pend = false;  // the previous unit's last P_1 V is still to be issued
        uint32_t pend_v = 0, pend_t = 0;
        bool pend_acc = false;
        auto flush = [&]() {
          if (!pend) return true;
          if (!pv_tile(1, pend_v % kSlots, pend_t, pend_acc)) return false;
          tc_commit(&kv_empty[pend_v % kSlots]);
          tc_commit(&o_full[1]);
          pend = false;
          return true;
        };
        for (int64_t u = blockIdx.x; ok && u < p.units; u += stride, ++it) {
          const Unit w = decode(p, u);
          const int n = w.nt;
          // tile 0
          uint32_t gk = g, gv = g + 1;
          if (!wait_q(0) || !wait_kv(gk)) break;
          qk(0, gk % kSlots);
          if (n == 1) free_q(0);
          if (!flush() || !wait_q(1)) break;
          qk(1, gk % kSlots);
          tc_commit(&kv_empty[gk % kSlots]);
          if (n == 1) free_q(1);
          if (!wait_kv(gv) || !wait_oe(0) || !pv_tile(0, gv % kSlots, tiles, false)) break;
          uint32_t prev_v = gv;
          g += 2;
          for (int i = 1; i < n; ++i) {
            gk = g;
            gv = g + 1;
            if (!wait_kv(gk)) break;
            qk(0, gk % kSlots);
            if (i == n - 1) free_q(0);
            if (i == 1 && !wait_oe(1)) break;
            if (!pv_tile(1, prev_v % kSlots, tiles + i - 1, i - 1 > 0)) break;
            tc_commit(&kv_empty[prev_v % kSlots]);
            qk(1, gk % kSlots);
            tc_commit(&kv_empty[gk % kSlots]);
            if (i == n - 1) free_q(1);
            if (!wait_kv(gv) || !pv_tile(0, gv % kSlots, tiles + i, true)) break;
            prev_v = gv;
            g += 2;
          }
          if (!ok) break;
          tc_commit(&o_full[0]);
          if (n == 1 && !wait_oe(1)) break;  // this unit's only P_1 V overwrites O_1
          pend = true;
          pend_v = prev_v;
          pend_t = tiles + n - 1;
          pend_acc = n > 1;
          tiles += n;
        }
        if (ok) flush();  // the last unit's last P_1 V
        tc_commit(mma_done);  // every MMA has completed before the tensor memory is freed
      }
      __syncwarp();
      {
        volatile int never = 0;
        mbar_wait(mma_done, 0, &never, globaltimer(), p.status, 39);
      }
      __syncwarp();
    }
  } else if (wg < 2) {
    setmaxnreg_inc<kSoftmaxRegs>();
    // ------------------------------------------------------------ softmax
    const int h = wg;                 // q head of the pair
    const int quad = warp & 3;        // tensor-memory lane quadrant of this warp
    const int r = quad * 32 + lane;   // query row within the block
    const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
    const uint32_t s_addr = tmem + lane_addr + kColS + 128 * h;
    const uint32_t o_addr = tmem + lane_addr + kColO + 128 * h;
    uint32_t t = 0, it = 0;
    for (int64_t u = blockIdx.x; u < p.units; u += stride, ++it) {
      const Unit w = decode(p, u);
      const int q0 = w.qb * kBlk, qi = q0 + r;
      float m = -INFINITY, l = 0.0f;
      bool ok = true;
      for (int i = 0; i < w.nt; ++i, ++t) {
        if (!(ok = warp_wait(&s_full[h], t & 1u, abort_flag, t0, p.status, 40 + h))) break;
        tc_fence_after();
        uint32_t sr[128];
        tmem_ld_32x32b_x32(s_addr + 0, *reinterpret_cast<uint32_t(*)[32]>(sr + 0));
        tmem_ld_32x32b_x32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
        tmem_ld_32x32b_x32(s_addr + 64, *reinterpret_cast<uint32_t(*)[32]>(sr + 64));
        tmem_ld_32x32b_x32(s_addr + 96, *reinterpret_cast<uint32_t(*)[32]>(sr + 96));
        tmem_ld_wait();
        float* s = reinterpret_cast<float*>(sr);
        const int k0 = key_tile(w, i) * kBlk;
        const bool band_full = p.window < 0 || (q0 + kBlk - 1 - k0 <= p.window && k0 + kBlk - 1 - q0 <= p.window);
        if (k0 + kBlk > p.L || !band_full) {  // mask keys past the end and outside the band
          int lo = 0, hi = min(kBlk - 1, p.L - 1 - k0);
          if (p.window >= 0) {
            lo = max(lo, qi - p.window - k0);
            hi = min(hi, qi + p.window - k0);
          }
          if (__any_sync(0xffffffffu, lo > 0)) {  // keys before the band
#pragma unroll
            for (int c = 0; c < 128; ++c) s[c] = c < lo ? -INFINITY : s[c];
          }
          if (__any_sync(0xffffffffu, hi < kBlk - 1)) {  // keys after the band or past the end
#pragma unroll
            for (int c = 0; c < 128; ++c) s[c] = c > hi ? -INFINITY : s[c];
          }
        }
        // row maximum: eight independent chains of three-input maxima
        float mc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          mc[j] = fmaxf(s[j], s[j + 8]);
#pragma unroll
          for (int t = 2; t < 16; t += 2) mc[j] = max3(mc[j], s[j + 8 * t], s[j + 8 * t + 8]);
        }
        const float mx = max3(max3(mc[0], mc[1], mc[2]), max3(mc[3], mc[4], mc[5]), fmaxf(mc[6], mc[7]));
        const float mt = mx * p.scale_log2;
        float factor = 1.0f;
        bool rescale = false;
        if (mt > m + kRescaleLog2 || (m == -INFINITY && mt > -INFINITY)) {
          factor = ex2(m - mt);  // 0 when m is still -inf
          rescale = (i > 0);
          l *= factor;
          m = mt;
        }
        const float mo = (m == -INFINITY) ? 0.0f : m;
        const float2 sc = make_float2(p.scale_log2, p.scale_log2), nm = make_float2(-mo, -mo);
        float2 acc[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                         make_float2(0.0f, 0.0f)};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (c == 2) {  // keys 0-63 published: their P V starts while keys 64-127 are computed
            if (__any_sync(0xffffffffu, rescale)) {
              // O_h *= factor before this tile's first P V (O_h is idle: see the MMA order
              // above); here half of the scores' registers are free for 32-column chunks
#pragma unroll
              for (int oc = 0; oc < 4; ++oc) {
                uint32_t o[32];
                tmem_ld_32x32b_x32(o_addr + 32 * oc, o);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * factor);
                tmem_st_32x32b_x32(o_addr + 32 * oc, o);
              }
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&pa_full[h]);
          }
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float2 x = fma_f2(make_float2(s[32 * c + 2 * j], s[32 * c + 2 * j + 1]), sc, nm);
            const float2 e = make_float2(ex2(x.x), ex2(x.y));
            acc[j & 3] = add_f2(acc[j & 3], e);
            pk[j] = pack_bf16x2(e.x, e.y);
          }
          tmem_st_32x32b_x16(s_addr + kColP + 16 * c, pk);
        }
        const float2 a01 = add_f2(acc[0], acc[1]), a23 = add_f2(acc[2], acc[3]);
        l += (a01.x + a23.x) + (a01.y + a23.y);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pb_full[h]);
      }
      if (!ok) break;
      // hand the row sums to the epilogue warps and go on with the next unit
      if (!warp_wait(&l_empty[h], (it & 1u) ^ 1u, abort_flag, t0, p.status, 44 + h)) break;
      st_shared_f32(lbuf + 4 * (h * 128 + r), l);
      __syncwarp();
      if (lane == 0) mbar_arrive(&l_full[h]);
    }
  } else {
    setmaxnreg_dec<kEpilogueRegs>();
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
    const uint32_t stg = sbase + offStg + quad * kWarpStg;
    uint32_t it = 0;
    bool stored = false;
    for (int64_t u = blockIdx.x; u < p.units; u += stride, ++it) {
      const Unit w = decode(p, u);
      const int q0 = w.qb * kBlk;
      bool ok = true;
      for (int h = 0; h < 2; ++h) {
        if (!(ok = warp_wait(&l_full[h], it & 1u, abort_flag, t0, p.status, 46 + h))) break;
        float lr;
        asm volatile("ld.shared.f32 %0, [%1];" : "=f"(lr) : "r"(lbuf + 4 * (h * 128 + r)) : "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&l_empty[h]);
        const float inv = lr > 0.0f ? 1.0f / lr : 0.0f;
        if (!(ok = warp_wait(&o_full[h], it & 1u, abort_flag, t0, p.status, 42 + h))) break;
        tc_fence_after();
        if (stored) {  // the previous store has finished reading the staging boxes
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
        }
        const uint32_t o_addr = tmem + lane_addr + kColO + 128 * h;
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // 32 columns at a time
          uint32_t o[32];
          tmem_ld_32x32b_x32(o_addr + 32 * c, o);
          tmem_ld_wait();
          if (c == 3) {  // O_h fully read: the next unit's P V may overwrite it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_empty[h]);
          }
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {  // 16-byte chunk j = 4 c + jj of the row: columns 8 j .. 8 j + 7
            const int j = 4 * c + jj;
            const float* f = reinterpret_cast<const float*>(o + 8 * jj);
            const uint32_t a = stg + (j >> 3) * 4096 + lane * 128 + (((j & 7) ^ (lane & 7)) << 4);
            st_shared_v4(a, pack_bf16x2(f[0] * inv, f[1] * inv), pack_bf16x2(f[2] * inv, f[3] * inv),
                         pack_bf16x2(f[4] * inv, f[5] * inv), pack_bf16x2(f[6] * inv, f[7] * inv));
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && q0 + quad * 32 < p.S) {
          for (int half = 0; half < 2; ++half)
            tma_store_3d(&tmO, stg + half * 4096, (w.h0 + h) * kD + half * 64, q0 + quad * 32, w.b);
          bulk_commit();
          stored = true;
        }
        stored = __shfl_sync(0xffffffffu, stored, 0);
      }
      if (!ok) break;
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 13) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace attn

namespace {

int attention_check(const DemonAttnArgs* a) {
  DEMON_CHECK_ARG(a != nullptr, "attention: null argument block");
  DEMON_CHECK_ARG(a->q && a->k && a->v && a->o, "attention: null q / k / v / o");
  DEMON_CHECK_ARG(a->head_dim == 128, "attention: head_dim must be 128 (got %d)", a->head_dim);
  DEMON_CHECK_ARG(a->B >= 0 && a->S >= 0 && a->L >= 1 && a->Hq >= 1 && a->Hk >= 1,
                  "attention: bad sizes B=%d S=%d L=%d Hq=%d Hk=%d", a->B, a->S, a->L, a->Hq, a->Hk);
  DEMON_CHECK_ARG(a->Hq % a->Hk == 0 && (a->Hq / a->Hk) % 2 == 0,
                  "attention: Hq / Hk must be an even integer (Hq=%d Hk=%d)", a->Hq, a->Hk);
  DEMON_CHECK_ARG(a->window >= -1, "attention: window must be -1 (none) or >= 0 (got %d)", a->window);
  DEMON_CHECK_ARG(a->window < 0 || a->S == a->L, "attention: a band needs S == L (S=%d L=%d)", a->S, a->L);
  DEMON_CHECK_ARG(a->scale > 0.0f, "attention: scale must be positive");
  const auto al16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  DEMON_CHECK_ARG(al16(a->q) && al16(a->k) && al16(a->v) && al16(a->o), "attention: pointers must be 16-byte aligned");
  DEMON_CHECK_ARG(a->ldq >= (int64_t)a->Hq * 128 && a->ldk >= (int64_t)a->Hk * 128 && a->ldv >= (int64_t)a->Hk * 128 &&
                      a->ldo >= (int64_t)a->Hq * 128,
                  "attention: row pitches must hold every head (ldq=%lld ldk=%lld ldv=%lld ldo=%lld)",
                  (long long)a->ldq, (long long)a->ldk, (long long)a->ldv, (long long)a->ldo);
  DEMON_CHECK_ARG(a->ldq % 8 == 0 && a->ldk % 8 == 0 && a->ldv % 8 == 0 && a->ldo % 8 == 0 && a->sq % 8 == 0 &&
                      a->sk % 8 == 0 && a->sv % 8 == 0 && a->so % 8 == 0,
                  "attention: row and sequence pitches must be multiples of 8 elements");
  DEMON_CHECK_ARG(a->sq >= (int64_t)a->S * a->ldq && a->so >= (int64_t)a->S * a->ldo && a->sk >= (int64_t)a->L * a->ldk &&
                      a->sv >= (int64_t)a->L * a->ldv,
                  "attention: sequence pitches must cover a whole sequence");
  DEMON_CHECK_ARG((int64_t)a->S < (1 << 30) && (int64_t)a->L < (1 << 30), "attention: sequence too long");
  return DEMON_OK;
}

std::atomic<uint64_t> g_attn_attr{0};

}  // namespace
}  // namespace demon

using namespace demon;

extern "C" int demon_attention(const DemonAttnArgs* a, void* stream) {
  DEMON_API_BEGIN();
  const int rc0 = attention_check(a);
  if (rc0 != DEMON_OK) return rc0;
  if (a->B == 0 || a->S == 0) return DEMON_OK;
  CUtensorMap tq, tk, tv, to;
  int rc;
  if ((rc = make_tmap_3d_bf16(&tq, a->q, (uint64_t)a->Hq * 128, (uint64_t)a->S, (uint64_t)a->B, (uint64_t)a->ldq * 2,
                              (uint64_t)a->sq * 2, 64, 128)) != DEMON_OK)
    return rc;
  if ((rc = make_tmap_3d_bf16(&tk, a->k, (uint64_t)a->Hk * 128, (uint64_t)a->L, (uint64_t)a->B, (uint64_t)a->ldk * 2,
                              (uint64_t)a->sk * 2, 64, 128)) != DEMON_OK)
    return rc;
  if ((rc = make_tmap_3d_bf16(&tv, a->v, (uint64_t)a->Hk * 128, (uint64_t)a->L, (uint64_t)a->B, (uint64_t)a->ldv * 2,
                              (uint64_t)a->sv * 2, 64, 128)) != DEMON_OK)
    return rc;
  if ((rc = make_tmap_3d_bf16(&to, a->o, (uint64_t)a->Hq * 128, (uint64_t)a->S, (uint64_t)a->B, (uint64_t)a->ldo * 2,
                              (uint64_t)a->so * 2, 64, 32)) != DEMON_OK)
    return rc;
  attn::Params p{};
  p.B = a->B;
  p.S = a->S;
  p.L = a->L;
  p.Hk = a->Hk;
  p.G = a->Hq / a->Hk;
  p.window = a->window;
  p.n_qblk = (a->S + attn::kBlk - 1) / attn::kBlk;
  p.n_kblk = (a->L + attn::kBlk - 1) / attn::kBlk;
  p.pairs = p.G / 2;
  p.scale_log2 = (float)((double)a->scale * 1.4426950408889634);
  p.units = (int64_t)a->B * a->Hk * p.pairs * p.n_qblk;
  DEMON_CHECK_ARG(p.units < ((int64_t)1 << 31), "attention: too many work units (%lld)", (long long)p.units);
  p.div_qblk = attn::make_fastdiv((uint32_t)p.n_qblk);
  p.div_pairs = attn::make_fastdiv((uint32_t)p.pairs);
  p.div_hk = attn::make_fastdiv((uint32_t)p.Hk);
  p.status = status_word();
  if (device_pending(g_attn_attr)) {
    // the warpgroups' register split is sized against the launch's 128 registers per thread;
    // with fewer at launch the softmax warps' setmaxnreg.inc would never return
    cudaFuncAttributes fa;
    DEMON_CUDA(cudaFuncGetAttributes(&fa, attn::attention_kernel));
    if (fa.numRegs != attn::kLaunchRegs) {
      set_error("attention: kernel built with %d registers per thread, the register split needs %d", fa.numRegs,
                attn::kLaunchRegs);
      return DEMON_ERR_CUDA;
    }
    DEMON_CUDA(cudaFuncSetAttribute(attn::attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, attn::kSmem));
    mark_device_done(g_attn_attr);
  }
  int dev = 0, sms = 148;
  DEMON_CUDA(cudaGetDevice(&dev));
  DEMON_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const unsigned grid = (unsigned)std::min<int64_t>(p.units, sms);
  attn::attention_kernel<<<grid, attn::kThreads, attn::kSmem, (cudaStream_t)stream>>>(tq, tk, tv, to, p);
  DEMON_CUDA(cudaGetLastError());
  return DEMON_OK;
}

extern "C" int64_t demon_attention_args_size(void) { return (int64_t)sizeof(DemonAttnArgs); }
