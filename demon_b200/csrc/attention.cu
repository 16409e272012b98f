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
// CTAs (one per SM) walk the units in a static round-robin.
//
// Warp roles (320 threads):
//   warps 0-3  softmax + epilogue of q head 0 of the unit (one query row per thread),
//   warps 4-7  the same for q head 1,
//   warp  8    TMA loads (Q pair, then K_i, V_i for each key tile into a 3-slot ring),
//   warp  9    MMA issue (one thread) and tensor-memory allocation.
// Tensor memory (512 columns): S_h at 128 h, O_h at 256 + 128 h (fp32, row = lane); P_h, the
// bf16 probabilities, overwrite the upper half of S_h (columns 128 h + 64 ..) and feed the
// P V MMA straight from tensor memory.  The MMAs of one thread run in issue order, which is
// what lets the next S_h = Q K^T overwrite P_h: it is issued after the P V that reads it.
//
// MMA order per unit with n key tiles (the S of one head is computed while the other head's
// softmax runs):
//   QK0(0) QK1(0) PV0(0) | for i >= 1: QK0(i) PV1(i-1) QK1(i) PV0(i) | PV1(n-1)
// The commit that signals S_h(i) therefore also covers PV_h(i-1): when a softmax warp sees
// S_h(i), no MMA touches O_h until it publishes P_h(i), so it may rescale O_h in place.
//
// Softmax (per row, log2 domain): t = s * scale * log2(e).  The running offset m is only
// raised when a tile's row maximum exceeds it by more than 8 (then O_h and the row sum are
// rescaled by 2^(m_old - m_new)); otherwise the stale offset stays, so p = 2^(t - m) <= 256.
// Numerator and denominator use the same offset, so the result is the exact softmax up to
// rounding (the lazy rescaling of FlashAttention-4, Dao et al. 2025).
//
// Epilogue: after the unit's last P V, each softmax warp reads its 32 rows of O_h from
// tensor memory, hands the columns back to the MMA warp, scales by 1 / rowsum, and stores
// the bf16 rows through a swizzled shared-memory box with its own TMA stores (rows past the
// sequence end are clipped by the tensor map).
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
constexpr int kSlots = 3;               // K / V ring slots
constexpr int kWarpStg = 2 * 32 * 128;  // one warp's 32-row O staging (two 4 KB boxes)
constexpr int kThreads = 320;

constexpr int offQ = 0;                                 // Q of both heads (64 KB)
constexpr int offKV = offQ + 2 * kTile;                 // ring (96 KB)
constexpr int offStg = offKV + kSlots * kTile;          // 8 warps x 8 KB
constexpr int offBar = offStg + 8 * kWarpStg;           // mbarriers
constexpr int kNumBars = 2 + 2 * kSlots + 2 * 4 + 1;
constexpr int offMisc = offBar + kNumBars * 8;          // tmem holder, abort flag
constexpr int kSmemUsed = offMisc + 16;
constexpr int kSmem = kSmemUsed + 1024;                 // + alignment slack
static_assert(kSmem <= 232448, "attention shared memory exceeds the sm_100 per-block limit");

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColP = 64, kColO = 256;  // S_h at 128 h, P_h at 128 h + 64, O_h at 256 + 128 h
constexpr float kRescaleLog2 = 8.0f;                    // lazy rescale threshold (log2 units)

struct Params {
  int B, S, L, Hk, G, window;  // window < 0: no band
  int n_qblk, n_kblk, pairs;   // blocks of 128 queries, tiles of 128 keys, q-head pairs per kv head
  float scale_log2;            // softmax scale * log2(e)
  int64_t units;
  unsigned int* status;
};

struct Unit {
  int b, hk, h0, qb, kt0, nt;  // sequence, kv head, first q head, query block, first key tile, tiles
};

__device__ __forceinline__ Unit decode(const Params& p, int64_t u) {
  Unit w;
  w.qb = (int)(u % p.n_qblk);
  int64_t r = u / p.n_qblk;
  const int pair = (int)(r % p.pairs);
  r /= p.pairs;
  w.hk = (int)(r % p.Hk);
  w.b = (int)(r / p.Hk);
  w.h0 = w.hk * p.G + 2 * pair;
  const int q0 = w.qb * kBlk;
  if (p.window >= 0) {
    const int qlast = min(q0 + kBlk - 1, p.S - 1);
    const int klo = max(0, q0 - p.window);
    const int khi = min(p.L - 1, qlast + p.window);
    w.kt0 = klo / kBlk;
    w.nt = khi / kBlk - w.kt0 + 1;
  } else {
    w.kt0 = 0;
    w.nt = p.n_kblk;
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

// Pairs of probabilities (within each group of eight pairs of a row) whose 2^x runs on the
// FMA pipe (exp2_poly2) instead of the MUFU unit, which alone would need as many cycles per
// key tile as the tensor core: bit j set = pair j of the group.
#ifndef DEMON_ATTN_POLY_PAIRS
#define DEMON_ATTN_POLY_PAIRS 0x88
#endif
constexpr unsigned kPolyPairs = DEMON_ATTN_POLY_PAIRS;

// 2^x for a pair, x <= 128, on the FMA pipe: range reduction x = j + r with j = rint(x)
// (Cody-Waite: adding 1.5 * 2^23 rounds to an integer in the low mantissa bits) and
// r in [-1/2, 1/2]; 2^r by a degree-3 polynomial whose coefficients are a relative-error
// minimax fit (Lawson's iteratively reweighted least squares, 4001 Chebyshev nodes; max
// relative error 7.5e-5 in fp32, below the bf16 rounding the probabilities get next); 2^j
// is added to the exponent field.  x is clamped at -126, where 2^x no longer matters next
// to the row's largest term (>= 1).
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  const float magic = 12582912.0f;  // 1.5 * 2^23
  x = make_float2(fmaxf(x.x, -126.0f), fmaxf(x.y, -126.0f));
  const float2 t = add_f2(x, make_float2(magic, magic));
  const float2 j = add_f2(t, make_float2(-magic, -magic));
  const float2 r = fma_f2(j, make_float2(-1.0f, -1.0f), x);
  float2 q = fma_f2(make_float2(0.0551716685f, 0.0551716685f), r, make_float2(0.2426111400f, 0.2426111400f));
  q = fma_f2(q, r, make_float2(0.6932609677f, 0.6932609677f));
  q = fma_f2(q, r, make_float2(0.9999280572f, 0.9999280572f));
  // bits(t) = bits(1.5 * 2^23) + j, whose low 9 bits are those of j; shifted by 23 the
  // constant part vanishes modulo 2^32, leaving j << 23
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

// A warp-uniform bounded wait: every lane waits, and the warp proceeds only if all did.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, uint64_t t0,
                                          unsigned int* status, unsigned int where) {
  const bool ok = mbar_wait(bar, parity, abort, t0, status, where);
  return __all_sync(0xffffffffu, ok && *abort == 0);
}

__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                     const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + offBar);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* kv_full = bars + 2;
  uint64_t* kv_empty = bars + 2 + kSlots;
  uint64_t* s_full = bars + 2 + 2 * kSlots;  // [2]
  uint64_t* p_full = s_full + 2;             // [2]
  uint64_t* o_full = s_full + 4;             // [2]
  uint64_t* o_empty = s_full + 6;            // [2]
  uint64_t* mma_done = s_full + 8;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + offMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + offMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t t0 = globaltimer();

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&s_full[h], 1);
      mbar_init(&p_full[h], 4);   // one arrive per softmax warp
      mbar_init(&o_full[h], 1);
      mbar_init(&o_empty[h], 4);  // one arrive per softmax warp
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8 && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmO);
  }
  if (warp == 9) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int64_t stride = gridDim.x;

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      uint32_t g = 0, it = 0, nq = 0;  // K / V tiles issued, units started, Q pairs issued
      bool ok = true;
      for (int64_t u = blockIdx.x; ok && u < p.units; u += stride, ++it) {
        const Unit w = decode(p, u);
        if (!(ok = mbar_wait(q_empty, (it & 1u) ^ 1u, abort_flag, t0, p.status, 21))) break;
        mbar_arrive_expect_tx(q_full, 2 * kTile);
        for (int h = 0; h < 2; ++h)
          for (int half = 0; half < 2; ++half)
            tma_load_3d(sbase + offQ + h * kTile + half * kBox, &tmQ, q_full, (w.h0 + h) * kD + half * 64,
                        w.qb * kBlk, w.b);
        ++nq;
        for (int i = 0; ok && i < w.nt; ++i) {
          const int k0 = (w.kt0 + i) * kBlk;
          for (int kv = 0; kv < 2; ++kv, ++g) {
            const int s = (int)(g % kSlots);
            if (!(ok = mbar_wait(&kv_empty[s], ((g / kSlots) & 1u) ^ 1u, abort_flag, t0, p.status, 22))) break;
            mbar_arrive_expect_tx(&kv_full[s], kTile);
            const CUtensorMap* m = kv ? &tmV : &tmK;
            for (int half = 0; half < 2; ++half)
              tma_load_3d(sbase + offKV + s * kTile + half * kBox, m, &kv_full[s], w.hk * kD + half * 64, k0, w.b);
          }
        }
      }
      // drain: no copy may still be in flight when the CTA leaves (immediate on the normal path)
      volatile int never = 0;
      for (uint32_t i = g > (uint32_t)kSlots ? g - kSlots : 0; i < g; ++i)
        mbar_wait(&kv_full[i % kSlots], (i / kSlots) & 1u, &never, globaltimer(), p.status, 23);
      if (nq) mbar_wait(q_full, (nq - 1) & 1u, &never, globaltimer(), p.status, 24);
    }
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      const uint32_t idesc_qk = idesc_bf16(kBlk, kBlk);
      const uint32_t idesc_pv = idesc_bf16(kBlk, kD) | (1u << 16);  // B (V) MN-major
      uint32_t g = 0, it = 0, tiles = 0;  // K / V tiles consumed, units, key tiles (all units)
      bool ok = true;
      auto qk = [&](int h, uint32_t kslot) {
        const uint32_t qa = sbase + offQ + h * kTile, kb = sbase + offKV + kslot * kTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_bf16(tmem + kColS + 128 * h, kmajor_desc(qa, kk), kmajor_desc(kb, kk), idesc_qk, kk > 0);
        tc_commit(&s_full[h]);
      };
      auto pv = [&](int h, uint32_t vslot, bool acc) {
        const uint32_t vb = sbase + offKV + vslot * kTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_bf16_ts(tmem + kColO + 128 * h, tmem + kColS + 128 * h + kColP + 8 * kk, mnmajor_desc(vb, kk),
                      idesc_pv, (acc || kk > 0) ? 1u : 0u);
      };
      auto wait_kv = [&](uint32_t gi) {
        ok = mbar_wait(&kv_full[gi % kSlots], (gi / kSlots) & 1u, abort_flag, t0, p.status, 31);
        if (ok) tc_fence_after();
        return ok;
      };
      auto wait_p = [&](int h, uint32_t t) {
        ok = mbar_wait(&p_full[h], t & 1u, abort_flag, t0, p.status, 32 + h);
        if (ok) tc_fence_after();
        return ok;
      };
      auto wait_oe = [&](int h) {
        ok = mbar_wait(&o_empty[h], (it & 1u) ^ 1u, abort_flag, t0, p.status, 34 + h);
        if (ok) tc_fence_after();
        return ok;
      };
      for (int64_t u = blockIdx.x; ok && u < p.units; u += stride, ++it) {
        const Unit w = decode(p, u);
        const int n = w.nt;
        if (!(ok = mbar_wait(q_full, it & 1u, abort_flag, t0, p.status, 30))) break;
        tc_fence_after();
        // tile 0
        uint32_t gk = g, gv = g + 1;
        if (!wait_kv(gk)) break;
        qk(0, gk % kSlots);
        qk(1, gk % kSlots);
        tc_commit(&kv_empty[gk % kSlots]);
        if (n == 1) tc_commit(q_empty);
        if (!wait_kv(gv) || !wait_oe(0) || !wait_p(0, tiles)) break;
        pv(0, gv % kSlots, false);
        uint32_t prev_v = gv;
        g += 2;
        for (int i = 1; i < n; ++i) {
          gk = g;
          gv = g + 1;
          if (!wait_kv(gk)) break;
          qk(0, gk % kSlots);
          if (i == 1 && !wait_oe(1)) break;
          if (!wait_p(1, tiles + i - 1)) break;
          pv(1, prev_v % kSlots, i - 1 > 0);
          tc_commit(&kv_empty[prev_v % kSlots]);
          qk(1, gk % kSlots);
          tc_commit(&kv_empty[gk % kSlots]);
          if (i == n - 1) tc_commit(q_empty);
          if (!wait_kv(gv) || !wait_p(0, tiles + i)) break;
          pv(0, gv % kSlots, true);
          prev_v = gv;
          g += 2;
        }
        if (!ok) break;
        tc_commit(&o_full[0]);
        if (n == 1 && !wait_oe(1)) break;
        if (!wait_p(1, tiles + n - 1)) break;
        pv(1, prev_v % kSlots, n > 1);
        tc_commit(&kv_empty[prev_v % kSlots]);
        tc_commit(&o_full[1]);
        tiles += n;
      }
      if (!ok) {  // wake the softmax warps on the abort path
        for (int h = 0; h < 2; ++h) {
          tc_commit(&s_full[h]);
          tc_commit(&o_full[h]);
        }
      }
      tc_commit(mma_done);  // every MMA has completed before the tensor memory is freed
    }
    __syncwarp();
    {
      volatile int never = 0;
      mbar_wait(mma_done, 0, &never, globaltimer(), p.status, 39);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int h = warp >> 2;          // q head of the pair
    const int quad = warp & 3;        // tensor-memory lane quadrant of this warp
    const int r = quad * 32 + lane;   // query row within the block
    const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
    const uint32_t s_addr = tmem + lane_addr + kColS + 128 * h;
    const uint32_t o_addr = tmem + lane_addr + kColO + 128 * h;
    const uint32_t stg = sbase + offStg + warp * kWarpStg;
    uint32_t t = 0, it = 0;
    bool stored = false;
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
        const int k0 = (w.kt0 + i) * kBlk;
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
        if (__any_sync(0xffffffffu, rescale)) {  // O_h is idle here (see the MMA order above)
#pragma unroll 1
          for (int c = 0; c < 16; ++c) {  // 8 columns at a time: the 128 scores stay in registers
            uint32_t o[8];
            tmem_ld_32x32b_x8(o_addr + 8 * c, o);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * factor);
            tmem_st_32x32b_x8(o_addr + 8 * c, o);
          }
        }
        const float mo = (m == -INFINITY) ? 0.0f : m;
        const float2 sc = make_float2(p.scale_log2, p.scale_log2), nm = make_float2(-mo, -mo);
        float2 acc[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                         make_float2(0.0f, 0.0f)};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float2 x = fma_f2(make_float2(s[32 * c + 2 * j], s[32 * c + 2 * j + 1]), sc, nm);
            const float2 e = ((kPolyPairs >> (j & 7)) & 1) ? exp2_poly2(x) : make_float2(ex2(x.x), ex2(x.y));
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
        if (lane == 0) mbar_arrive(&p_full[h]);
      }
      if (!ok) break;
      // ---- epilogue: O_h rows of this warp -> bf16, 1 / rowsum, TMA store
      if (!warp_wait(&o_full[h], it & 1u, abort_flag, t0, p.status, 42 + h)) break;
      tc_fence_after();
      uint32_t o[128];
      tmem_ld_32x32b_x32(o_addr + 0, *reinterpret_cast<uint32_t(*)[32]>(o + 0));
      tmem_ld_32x32b_x32(o_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
      tmem_ld_32x32b_x32(o_addr + 64, *reinterpret_cast<uint32_t(*)[32]>(o + 64));
      tmem_ld_32x32b_x32(o_addr + 96, *reinterpret_cast<uint32_t(*)[32]>(o + 96));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[h]);
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      if (stored) {  // the previous unit's store has finished reading the staging boxes
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {  // 16-byte chunk j of the row: columns 8 j .. 8 j + 7
        const float* f = reinterpret_cast<const float*>(o + 8 * j);
        const uint32_t a = stg + (j >> 3) * 4096 + lane * 128 + (((j & 7) ^ (lane & 7)) << 4);
        st_shared_v4(a, pack_bf16x2(f[0] * inv, f[1] * inv), pack_bf16x2(f[2] * inv, f[3] * inv),
                     pack_bf16x2(f[4] * inv, f[5] * inv), pack_bf16x2(f[6] * inv, f[7] * inv));
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
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, kTmemCols);
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
  p.status = status_word();
  if (device_pending(g_attn_attr)) {
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
