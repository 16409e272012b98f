// nvfp4_gemm.cu -- tcgen05 block-scaled NVFP4 GEMM with fused epilogue (sm_100a),
// and the bf16 tcgen05 GEMM used for the LoRA down-projection.
//
// Persistent kernel: one CTA per SM (for N % 256 == 0 a 2-CTA cluster per SM pair, cta_group::2
// MMAs on 256 x 256 tiles) walks output tiles in bands of m-blocks swept over N (or, for the
// rotary side tile, contiguous tiles with N fastest).  Warp roles (384 threads, three
// warpgroups; setmaxnreg gives the first 56 registers per thread and the other two 224):
//   warp 0      TMA producer: A/B tiles with tiled TMA loads (128-byte swizzle, no
//               multicast) and the stage's block scales -- the quantiser writes scales in
//               the tcgen05 128x4-chunk layout, so a stage's scales are contiguous.  It runs
//               ahead into the next tile while the epilogue drains the current one.
//   warp 1      TMEM allocation + one MMA-issuing thread: per stage it copies the scales
//               SMEM -> TMEM (tcgen05.cp 32x128b.warpx4, replicated into the four lane
//               quadrants), issues four tcgen05.mma.kind::mxf4nvf4.block_scale.block16
//               (K = 64 each) and commits to the stage's "empty" barrier.
//   warp 2      side-input loader (SIDE 1 / 2): the rotary table rows or the residual tile
//               (with the tile's gate rows) into shared memory, so that the epilogue reads
//               its per-row operands from there and not one row per lane from global memory.
//   warp 3      idle.
//   warps 4-11  epilogue, two warps per TMEM lane quadrant, each owning half of the tile's
//               columns.  Per-column vectors and row scales are fetched while the MMAs run;
//               the warps drain their accumulator columns with tcgen05.ld and release TMEM at
//               once (the MMA warp starts the next tile), convert each row to bf16 (alpha *
//               acc + bias, one rounding), apply head norm + RoPE, SwiGLU, gate and residual in
//               bf16 as the reference's eager ops do, and write 32x32 blocks through a
//               double-buffered, 64-byte-swizzled staging area with TMA stores (the residual
//               mode writes over the staged residual and stores 32x64 boxes from there).
// Modes (the SIDE template argument, chosen per call on the host): 0 plain (4 stages), 1 the
// rotary side tile, 2 the residual side tile, 3 no per-column vector (no bias: 5 stages), 5 as
// 3 with the bias read from global memory.  Pair launches allow programmatic dependent launch.
// Hot LoRA: for each 64-wide slice of the rank, one extra pipeline stage holds
// the xa tile (128 x 64 bf16, 16 KB -- the size of an A stage) and the
// lora_b tile (BN x 64 bf16 -- the size of a B stage); four kind::f16 MMAs
// accumulate xa . lora_b^T into the same TMEM accumulator before the FP4
// K-loop.  xa is pre-divided by alpha and pre-multiplied by the strength
// (demon_lora_down), so a strength change never touches the packed weights.
//
// Every mbarrier wait is bounded (demon_common.cuh); on expiry the CTA records
// DEMON_DEV_TIMEOUT, stops issuing, drains what it issued and frees TMEM.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "demon_common.cuh"
#include "demon_host.h"

namespace demon {

struct GemmParams {
  const uint8_t* a_sf;
  const uint8_t* w_sf;
  const float* a_gs;
  const float* w_gs;
  const float* col_scale;  // bf16 mode: per-output-column scale
  const __nv_bfloat16* bias;
  const __nv_bfloat16* gate;
  const __nv_bfloat16* residual;
  __nv_bfloat16* out;
  unsigned int* status;
  int64_t gate_rows, ld_gate, ldo, ldr;
  int M, N, K;
  int a_gs_per_row;
  int w_gs_per_block;  // w_gs[n / 128] instead of w_gs[0]
  int lora_rank;
  // per-head RMSNorm (+ RoPE) epilogue: heads of 128 in columns [0, hn_cols)
  int hn_cols, hn_q_cols;
  int64_t rope_S;
  const __nv_bfloat16* hn_wq;
  const __nv_bfloat16* hn_wk;
  const __nv_bfloat16* rope_cos;
  const __nv_bfloat16* rope_sin;
  float hn_eps;
  int m_tiles, n_tiles;
  int m_group;  // tile order: bands of m_group m-blocks, each swept over every n-block
  // > 0: CTA (pair) c takes the contiguous tiles [c * tile_chunk, (c + 1) * tile_chunk) instead
  // of every ncl-th tile; with m_group = 1 it sweeps N over one m-block before the next
  int tile_chunk;
  int silu_mul;  // SwiGLU epilogue: interleaved gate/up blocks of 128 -> h of width N / 2
  // bounded-wait test (demon_test_arm_gemm_stall): the first CTA (pair) waits at most wait_ns
  // and its rank-0 CTA withholds the loads of its first stage; 0 in normal launches
  int withhold;
  uint64_t wait_ns;
  int out_evict_first;  // output larger than L2: store it with an evict-first L2 policy
};

constexpr int kBM = 128;
constexpr int kRowBytes = 128;   // one 128-byte swizzle row per stage (256 fp4 / 64 bf16)
constexpr int kEpiWarps = 8;
// Warpgroup 0: the TMA producer (warp 0), the MMA issuer (warp 1) and two idle warps; warpgroups
// 1-2: the epilogue.  setmaxnreg moves registers from warpgroup 0 to the epilogue, whose loads of
// the gate, residual and rotary tables are kept in flight a step ahead of their use:
// 128 * 56 + 256 * 224 = 64,512 = 384 * 168, the launch's registers.
constexpr int kThreads = 128 + 32 * kEpiWarps;
constexpr int kGemmLaunchRegs = 168, kGemmIssueRegs = 56, kGemmEpiRegs = 224;
static_assert(128 * kGemmIssueRegs + 32 * kEpiWarps * kGemmEpiRegs <= kThreads * kGemmLaunchRegs,
              "register split exceeds the launch's registers (setmaxnreg.inc would wait for good)");
constexpr int kStgPitch = 80;     // bf16-GEMM transpose staging: 32 bf16 + 16 bytes of padding per row

// SIDE: 0 no side tile, 1 the rotary tables (head norm + RoPE), 2 the residual (no bias), 3
// none and no per-column vector either (no bias: the space goes to a fifth stage), 5 as 3 with
// the bias read from global memory in the epilogue (a separate kernel: 3's code stays as it is)
template <int BN, int STAGES, bool FP4, bool PAIR = false, int SIDE = 0>
struct GemmCfg {
  static constexpr bool kSideTile = SIDE == 1 || SIDE == 2;
  static constexpr bool kColVec = SIDE == 0 || SIDE == 1;  // bias / column scale staged per warp
  static constexpr int kA = kBM * kRowBytes;
  static constexpr int kB = (PAIR ? BN / 2 : BN) * kRowBytes;  // a CTA pair splits the B tile
  static constexpr int kSFA = FP4 ? 2048 : 0;
  static constexpr int kSFB = FP4 ? ((BN + 127) / 128) * 2048 : 0;
  static constexpr int offA = 0;
  static constexpr int offB = offA + STAGES * kA;
  static constexpr int offSFA = offB + STAGES * kB;
  static constexpr int offSFB = offSFA + STAGES * kSFA;
  // per epilogue warp: two 2 KB TMA-store staging buffers (FP4), or one transpose block (bf16);
  // none with the residual side tile, whose rows the output overwrites and is stored from
  static constexpr int kStgWarp = SIDE == 2 ? 0 : FP4 ? 4096 : 32 * kStgPitch;
  static constexpr int offStg = (offSFB + STAGES * kSFB + 1023) / 1024 * 1024;
  // side-input tile (SIDE kernels), loaded by a loader warp and read row by row: the rotary
  // tables of the CTA's 128 rows (tables with equal halves: per row the 64-column cos half and
  // the sin half, 256 bytes at a 272-byte pitch, so that a warp's row-per-lane 16-byte reads
  // are conflict-free), or the residual tile (four 128-row x 64-column TMA boxes with the
  // 128-byte swizzle) and the tile's segments of the (at most two) gate rows its 128 rows use
  static constexpr int kSideRow = 272;
  static constexpr int kSideGate = 4 * kBM * 128;  // offset of the gate segments (SIDE 2)
  // (SIDE 2: then one int, the first row of the tile's second gate row)
  static constexpr int kSide = SIDE == 1 ? kBM * kSideRow : SIDE == 2 ? kSideGate + 2 * BN * 2 + 16 : 0;
  static constexpr int offSide = offStg + kEpiWarps * kStgWarp;  // 1024-aligned (SW128 boxes)
  static constexpr int offCol = offSide + kSide;                 // fp32 per-column vector per warp
  static constexpr int offHn = offCol + (kColVec ? kEpiWarps * (BN / 2) * 4 : 0);
  // head-norm weight per warp: its 128 columns as 64 bf16 pairs
  static constexpr int offBar = offHn + (FP4 && SIDE != 2 ? kEpiWarps * (BN / 2) * 2 : 0);
  static constexpr int kBars = 2 * STAGES + 3 + (kSideTile ? 2 : 0);
  static constexpr int offMisc = offBar + kBars * 8;
  static constexpr int kSmem = offMisc + 16 + 1024;  // + alignment slack
  static constexpr int kSfaCol = BN;                 // 4 columns per K=64 step, 4 steps
  static constexpr int kSfbCol = BN + 16;            // ((BN+127)/128)*4 columns per step
  static constexpr int kUsedCols = FP4 ? BN + 16 + ((BN + 127) / 128) * 16 : BN;
  static constexpr uint32_t kTmemCols = kUsedCols <= 32 ? 32 : kUsedCols <= 64 ? 64 : kUsedCols <= 128 ? 128
                                        : kUsedCols <= 256 ? 256 : 512;
  static constexpr int kStepElems = FP4 ? 256 : 64;  // K elements per stage
  static constexpr int kColsPerWarp = BN / 2;        // columns per epilogue warp
  static constexpr int kChunks = kColsPerWarp / 32;  // 32-column chunks per epilogue warp
  static_assert(kSmem <= 232448, "shared memory budget");
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN");
  static_assert(!SIDE || (FP4 && BN == 256 && PAIR && offSide % 1024 == 0), "side tile");
};

// Tile t -> (m_blk, n_blk).  Tiles run in bands of m_group m-blocks: inside a band the
// m-block varies fastest, then the n-block, so the CTAs working at one time share a band
// of A rows (which stays in L2 while the band sweeps N) and a few B column blocks.  With
// m_group = m_tiles this is plain m-fastest order.
__device__ __forceinline__ void tile_coords(int t, const GemmParams& p, int& m_blk, int& n_blk) {
  const int band = p.m_group * p.n_tiles;
  const int b = t / band, j = t - b * band;
  const int gm = min(p.m_group, p.m_tiles - b * p.m_group);
  m_blk = b * p.m_group + j % gm;
  n_blk = j / gm;
}

__device__ __forceinline__ uint64_t sw128_desc(const void* p) {
  // K-major, 128-byte swizzle: 8-row core groups 1024 bytes apart.
  return smem_desc(smem_u32(p), 16, 1024, 2);
}
__device__ __forceinline__ uint64_t sf_desc(const void* p) {
  // 32 rows x 16 bytes, no swizzle: 8-row core matrices 128 bytes apart.
  return smem_desc(smem_u32(p), 0, 128, 0);
}
// Byte offset of 16-byte chunk j of row r in a 32 x 64-byte staging block with
// the TMA 64-byte swizzle (address bits [4,5] ^= bits [7,8]).
__device__ __forceinline__ int stg_off(int r, int j) { return r * 64 + ((j ^ ((r >> 1) & 3)) << 4); }

// One CTA per SM (persistent).  10 warps spread over the SM's 4 sub-partitions put 3 warps on
// two of them, so a thread gets at most 168 of a sub-partition's 16 K registers.
template <int BN, int STAGES, bool FP4, bool PAIR, int SIDE>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmLA, const __grid_constant__ CUtensorMap tmLB,
                const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmSFA,
                const __grid_constant__ CUtensorMap tmSFB, const __grid_constant__ CUtensorMap tmR,
                const GemmParams p) {
  using C = GemmCfg<BN, STAGES, FP4, PAIR, SIDE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::offBar);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* mma_done = acc_empty + 1;
  uint64_t* side_full = mma_done + 1;   // side-tile kernels only
  uint64_t* side_empty = mma_done + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::offMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::offMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // programmatic dependent launch: the next kernel in the stream may be scheduled now (it can only
  // use SMs this grid leaves, and it waits for this grid to complete before touching memory)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int KT = p.K / C::kStepElems;
  const int lboxes = p.lora_rank > 0 ? (p.lora_rank + 63) / 64 : 0;
  const int num_tiles = p.m_tiles * p.n_tiles;
  const uint64_t t0 = globaltimer();
  // CTA pair (cta_group::2): the pair computes a 256 x BN tile, CTA `rank` owns rows
  // 128 * rank .. +128 of it and half of the B tile; the leader (rank 0) issues the MMAs.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int cid = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int ncl = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  constexpr int kTileM = PAIR ? 2 * kBM : kBM;
  // this CTA's tiles: t_begin, t_begin + t_step, ... < t_end (every role walks the same list)
  const int t_begin = p.tile_chunk ? cid * p.tile_chunk : cid;
  const int t_step = p.tile_chunk ? 1 : ncl;
  const int t_end = p.tile_chunk ? min(num_tiles, t_begin + p.tile_chunk) : num_tiles;
  // Side-tile kernels: the side tile a tile reads, as a key (-1: none).  The rotary tables depend
  // on the rows only, so consecutive tiles of one m-block share one load; a residual tile is
  // its own.  A side tile is released after the last of a run of tiles with its key.
  auto side_key = [&](int tile) -> int {
    if (!C::kSideTile || tile >= t_end) return -1;
    int mb, nb;
    tile_coords(tile, p, mb, nb);
    if (SIDE == 1) return nb * BN < p.hn_cols ? mb : -1;
    return tile;
  };
  // wait limit of this CTA: the default, or the armed test's short one in the first CTA (pair)
  const uint64_t lim = (p.withhold && cid == 0) ? p.wait_ns : (uint64_t)DEMON_WAIT_LIMIT_NS;
  const bool hold0 = p.withhold && cid == 0 && rank == 0;  // test: skip the loads of stage 0

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, PAIR ? 2 * kEpiWarps : kEpiWarps);  // the pair's epilogue warps
    mbar_init(mma_done, 1);
    if (C::kSideTile) {
      mbar_init(side_full, 1);
      mbar_init(side_empty, kEpiWarps);  // this CTA's epilogue warps
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (lboxes) {
      prefetch_tmap(&tmLA);
      prefetch_tmap(&tmLB);
    }
    if (PAIR) {
      prefetch_tmap(&tmSFA);
      prefetch_tmap(&tmSFB);
    }
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(tmem_holder, C::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, C::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if (PAIR)
    cluster_sync();  // both CTAs' barriers are initialised before any remote arrive / complete_tx
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // the set-up above (barriers, tensor memory, tensor-map prefetch) overlaps the previous kernel's
  // tail; every global read and write comes after that kernel has completed
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (warp < 4) {
   asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kGemmIssueRegs));
   if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      uint32_t g = 0;  // stages issued so far (all tiles)
      const int64_t kchunks = p.K / 64;
      bool ok = true;
      for (int tile = t_begin; ok && tile < t_end; tile += t_step) {
        int m_blk, n_blk;
        tile_coords(tile, p, m_blk, n_blk);
        const int m0 = m_blk * kTileM, n0 = n_blk * BN;
        const int am0 = m0 + (int)rank * kBM;                  // this CTA's A rows
        const int bn0 = n0 + (int)rank * (BN / 2) * (PAIR ? 1 : 0);  // this CTA's B rows
        // a pair's stage completes on the leader's barrier with both CTAs' bytes
        const uint32_t mult = PAIR ? 2u : 1u;
        for (int b = 0; b < lboxes; ++b, ++g) {
          const int s = g % STAGES;
          if (!(ok = mbar_wait(&empty[s], ((g / STAGES) & 1u) ^ 1u, abort_flag, t0, p.status, 1, lim))) break;
          if (leader) mbar_arrive_expect_tx(&full[s], mult * (uint32_t)(C::kA + C::kB));
          if (hold0 && g == 0) continue;  // test: these bytes never arrive
          if (PAIR) {
            tma_load_2d_pair(smem + C::offA + s * C::kA, &tmLA, &full[s], b * 64, am0);
            tma_load_2d_pair(smem + C::offB + s * C::kB, &tmLB, &full[s], b * 64, bn0);
          } else {
            tma_load_2d(smem + C::offA + s * C::kA, &tmLA, &full[s], b * 64, am0);
            tma_load_2d(smem + C::offB + s * C::kB, &tmLB, &full[s], b * 64, bn0);
          }
        }
        // scale halves of the B tile that exist in the (128-row padded) scale buffer
        const int sfb_halves = FP4 ? std::min((BN + 127) / 128, (p.N - n0 + 127) / 128) : 0;
        const uint32_t tx = (uint32_t)(C::kA + C::kB + C::kSFA + sfb_halves * 2048);
        for (int kt = 0; ok && kt < KT; ++kt, ++g) {
          const int s = g % STAGES;
          if (!(ok = mbar_wait(&empty[s], ((g / STAGES) & 1u) ^ 1u, abort_flag, t0, p.status, 2, lim))) break;
          if (leader) mbar_arrive_expect_tx(&full[s], mult * tx);
          if (hold0 && g == 0) continue;  // test: these bytes never arrive
          const int kx = FP4 ? kt * kRowBytes : kt * 64;
          if (PAIR) {
            tma_load_2d_pair(smem + C::offA + s * C::kA, &tmA, &full[s], kx, am0);
            tma_load_2d_pair(smem + C::offB + s * C::kB, &tmB, &full[s], kx, bn0);
            if (FP4) {  // scale chunks through 256-byte-row views of the scale buffers (2 KB boxes)
              tma_load_2d_pair(smem + C::offSFA + s * C::kSFA, &tmSFA, &full[s], 0,
                               (int)(((int64_t)(am0 / kBM) * kchunks + kt * 4) * 2));
              for (int h = 0; h < sfb_halves; ++h)
                tma_load_2d_pair(smem + C::offSFB + s * C::kSFB + h * 2048, &tmSFB, &full[s], 0,
                                 (int)(((int64_t)(n0 / 128 + h) * kchunks + kt * 4) * 2));
            }
          } else {
            tma_load_2d(smem + C::offA + s * C::kA, &tmA, &full[s], kx, am0);
            tma_load_2d(smem + C::offB + s * C::kB, &tmB, &full[s], kx, bn0);
            if (FP4) {
              bulk_load(smem + C::offSFA + s * C::kSFA, p.a_sf + ((int64_t)m_blk * kchunks + kt * 4) * 512, 2048,
                        &full[s]);
              for (int h = 0; h < sfb_halves; ++h)
                bulk_load(smem + C::offSFB + s * C::kSFB + h * 2048,
                          p.w_sf + ((int64_t)(n_blk * ((BN + 127) / 128) + h) * kchunks + kt * 4) * 512, 2048,
                          &full[s]);
            }
          }
        }
      }
      // drain: never leave the CTA with copies in flight (returns at once on the normal path);
      // a pair's copies all complete on the leader's barriers, which the leader drains
      if (!leader) g = 0;
      for (uint32_t i = g > (uint32_t)STAGES ? g - STAGES : 0; i < g; ++i) {
        volatile int never = 0;
        mbar_wait(&full[i % STAGES], (i / STAGES) & 1u, &never, globaltimer(), p.status, 3, lim);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (pair leader)
    if (elect_one() && leader) {
      const uint32_t idesc = FP4 ? idesc_mxf4nvf4(kTileM, BN) : idesc_bf16(kTileM, BN);
      const uint32_t ib = idesc_bf16(kTileM, BN);
      uint32_t g = 0, it = 0;
      bool ok = true;
      for (int tile = t_begin; ok && tile < t_end; tile += t_step, ++it) {
        // the epilogue must have drained the previous tile's accumulator; without hot LoRA the
        // first stage's scale-factor copies are issued before that wait
        const bool early_sf = FP4 && lboxes == 0;
        if (!early_sf) {
          if (!(ok = mbar_wait(acc_empty, (it & 1u) ^ 1u, abort_flag, t0, p.status, 4, lim))) break;
          tc_fence_after();
        }
        uint32_t accum = 0;
        for (int b = 0; b < lboxes; ++b, ++g) {
          const int s = g % STAGES;
          if (!(ok = mbar_wait(&full[s], (g / STAGES) & 1u, abort_flag, t0, p.status, 5, lim))) break;
          tc_fence_after();
          const uint64_t la = sw128_desc(smem + C::offA + s * C::kA);
          const uint64_t lb = sw128_desc(smem + C::offB + s * C::kB);
          for (int j = 0; j < 4; ++j) {
            if (b * 64 + j * 16 < p.lora_rank) {
              if (PAIR)
                mma_bf16_pair(tmem, la + 2 * j, lb + 2 * j, ib, accum);
              else
                mma_bf16(tmem, la + 2 * j, lb + 2 * j, ib, accum);
              accum = 1;
            }
          }
          if (PAIR)
            tc_commit_pair(&empty[s]);
          else
            tc_commit(&empty[s]);
        }
        for (int kt = 0; ok && kt < KT; ++kt, ++g) {
          const int s = g % STAGES;
          if (!(ok = mbar_wait(&full[s], (g / STAGES) & 1u, abort_flag, t0, p.status, 6, lim))) break;
          tc_fence_after();
          const uint64_t adesc = sw128_desc(smem + C::offA + s * C::kA);
          const uint64_t bdesc = sw128_desc(smem + C::offB + s * C::kB);
          if (FP4) {
            const uint8_t* sfa = smem + C::offSFA + s * C::kSFA;
            const uint8_t* sfb = smem + C::offSFB + s * C::kSFB;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              // a pair copies each CTA's scale chunks (same offsets) into its own TMEM
              if (PAIR)
                tc_cp_32x128b_warpx4_pair(tmem + C::kSfaCol + 4 * j, sf_desc(sfa + j * 512));
              else
                tc_cp_32x128b_warpx4(tmem + C::kSfaCol + 4 * j, sf_desc(sfa + j * 512));
#pragma unroll
              for (int h = 0; h < (BN + 127) / 128; ++h) {
                if (PAIR)
                  tc_cp_32x128b_warpx4_pair(tmem + C::kSfbCol + ((BN + 127) / 128) * 4 * j + 4 * h,
                                            sf_desc(sfb + h * 2048 + j * 512));
                else
                  tc_cp_32x128b_warpx4(tmem + C::kSfbCol + ((BN + 127) / 128) * 4 * j + 4 * h,
                                       sf_desc(sfb + h * 2048 + j * 512));
              }
            }
            if (early_sf && kt == 0) {
              if (!(ok = mbar_wait(acc_empty, (it & 1u) ^ 1u, abort_flag, t0, p.status, 4, lim))) break;
              tc_fence_after();
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (PAIR)
                mma_mxf4nvf4_pair(tmem, adesc + 2 * j, bdesc + 2 * j, idesc, tmem + C::kSfaCol + 4 * j,
                                  tmem + C::kSfbCol + ((BN + 127) / 128) * 4 * j, accum);
              else
                mma_mxf4nvf4(tmem, adesc + 2 * j, bdesc + 2 * j, idesc, tmem + C::kSfaCol + 4 * j,
                             tmem + C::kSfbCol + ((BN + 127) / 128) * 4 * j, accum);
              accum = 1;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (PAIR)
                mma_bf16_pair(tmem, adesc + 2 * j, bdesc + 2 * j, idesc, accum);
              else
                mma_bf16(tmem, adesc + 2 * j, bdesc + 2 * j, idesc, accum);
              accum = 1;
            }
          }
          if (PAIR)
            tc_commit_pair(&empty[s]);
          else
            tc_commit(&empty[s]);
        }
        if (PAIR)
          tc_commit_pair(acc_full);
        else
          tc_commit(acc_full);
      }
      if (!ok) {  // wake the epilogue on the abort path
        if (PAIR)
          tc_commit_pair(acc_full);
        else
          tc_commit(acc_full);
      }
      // every MMA has completed before anyone frees TMEM
      if (PAIR)
        tc_commit_pair(mma_done);
      else
        tc_commit(mma_done);
    }
    if (lane == 0) {  // both CTAs of a pair learn of the last MMA through their own barrier
      volatile int never = 0;
      mbar_wait(mma_done, 0, &never, globaltimer(), p.status, 9, lim);
    }
    __syncwarp();
   } else if (C::kSideTile && warp == 2) {
    // ------------------------------------------------------------ side-input loader
    // At the first tile of each run of tiles with one side key, once the epilogue warps have
    // released the previous side tile: the table rows of the m-block by coalesced 16-byte
    // cp.async copies, half a warp per row (the cos and sin halves; positions wrap at rope_S
    // inside a tile; rows past M are skipped), or the residual tile by four TMA boxes (rows
    // past M read as zeros).
    constexpr bool side_rope = SIDE == 1;
    uint8_t* side = smem + C::offSide;
    uint32_t sit = 0;  // side tiles issued
    int loaded = -1;   // key of the side tile in shared memory (-1: released)
    for (int tile = t_begin; tile < t_end; tile += t_step) {
      const int key = side_key(tile);
      if (key < 0) continue;
      const bool fresh = key != loaded;
      loaded = side_key(tile + t_step) == key ? key : -1;  // the epilogue releases at a run's end
      if (!fresh) continue;
      int m_blk, n_blk;
      tile_coords(tile, p, m_blk, n_blk);
      const int m0 = m_blk * kTileM + (int)rank * kBM, n0 = n_blk * BN;
      if (!mbar_wait(side_empty, (sit & 1u) ^ 1u, abort_flag, t0, p.status, 10, lim)) break;
      if (side_rope) {
        const int rows = max(0, min(kBM, p.M - m0));
        const int hl = lane >> 4, ch = lane & 15;  // row parity, 16-byte chunk of the staged row
        const uint32_t sb = smem_u32(side);
        const __nv_bfloat16* tab = (ch < 8 ? p.rope_cos : p.rope_sin) + (ch & 7) * 8;
        int64_t pos = ((int64_t)m0 + hl) % p.rope_S;
        for (int r = hl; r < rows; r += 2) {
          cp_async_16(sb + r * C::kSideRow + ch * 16, tab + pos * 128);
          pos += 2;
          while (pos >= p.rope_S) pos -= p.rope_S;
        }
        cp_async_mbar_arrive(side_full);  // every lane's copies are part of this phase
        __syncwarp();
        if (lane == 0) mbar_arrive(side_full);
      } else if (lane == 0) {
        // gate rows of this CTA's rows inside M (gate_rows >= 128: one or two)
        const int g0 = m0 / (int)p.gate_rows;
        const int ng = (p.gate && m0 < p.M) ? (min(m0 + kBM, p.M) - 1) / (int)p.gate_rows - g0 + 1 : 0;
        // the epilogue's split between the two gate rows, published by the arrive below
        *reinterpret_cast<int*>(side + C::kSideGate + 2 * BN * 2) = (g0 + 1) * (int)p.gate_rows;
        mbar_arrive_expect_tx(side_full, 4u * kBM * 128u + (uint32_t)ng * (BN * 2));
        for (int b = 0; b < 4; ++b) tma_load_2d(side + b * (kBM * 128), &tmR, side_full, n0 + 64 * b, m0);
        for (int i = 0; i < ng; ++i)
          bulk_load(side + C::kSideGate + i * (BN * 2), p.gate + (int64_t)(g0 + i) * p.ld_gate + n0, BN * 2, side_full);
      }
      __syncwarp();
      ++sit;
    }
    // the CTA leaves only after its last side copy has landed (it may not have been read)
    if (sit > 0) {
      volatile int never = 0;
      mbar_wait(side_full, (sit - 1u) & 1u, &never, globaltimer(), p.status, 11, lim);
    }
    __syncwarp();
   }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kGemmEpiRegs));
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 4;            // 0..7
    const int q = warp & 3;             // TMEM lane quadrant accessible to this warp
    const int half = ew >> 2;           // which half of the tile's columns
    const uint32_t stg = smem_u32(smem + C::offStg + ew * C::kStgWarp);
    const uint32_t colv = smem_u32(smem + C::offCol) + ew * (C::kColsPerWarp * 4);
    const uint32_t hnv = smem_u32(smem + C::offHn) + ew * (C::kColsPerWarp * 2);
    if (FP4 && lane == 0) prefetch_tmap(&tmO);
    const uint64_t out_policy = l2_policy_evict_first();
    uint32_t it = 0, nstore = 0;
    // side-tile kernels: the rotary tables (head norm + RoPE) or the residual come from the side tile
    constexpr bool side_rope = SIDE == 1;
    constexpr bool side_res = SIDE == 2;
    const uint32_t side = smem_u32(smem + C::offSide);
    uint32_t sit = 0;  // side tiles released
    int cur = -1;      // key of the side tile this warp has seen land (-1: none)
    // SwiGLU: a BN = 256 tile holds gate block n and up block n of the interleaved weight; each
    // warp takes 64 output columns (its 64 gate and the matching 64 up accumulator columns)
    const bool sm = FP4 && BN == 256 && p.silu_mul != 0;
    for (int tile = t_begin; tile < t_end; tile += t_step, ++it) {
      int m_blk, n_blk;
      tile_coords(tile, p, m_blk, n_blk);
      const int m0 = m_blk * kTileM + (int)rank * kBM, n0 = n_blk * BN;  // this CTA's 128 rows
      const int ncol0 = n0 + half * C::kColsPerWarp;
      const int skey = side_key(tile);
      const bool need_side = skey >= 0;
      // Everything that does not depend on the accumulator is fetched while the MMAs run:
      // the per-column vector (bias, or the bf16 GEMM's column scale) into shared memory,
      // the lane's row scale, and L2 prefetches of its gate / residual row segments.
      for (int i = lane; C::kColVec && i < C::kColsPerWarp; i += 32) {
        const int n = sm ? n0 + (i < 64 ? half * 64 + i : 128 + half * 64 + (i - 64)) : ncol0 + i;
        float cv = 0.0f;
        if (n < p.N)
          cv = (FP4 || !p.col_scale) ? (p.bias ? __bfloat162float(p.bias[n]) : 0.0f) : p.col_scale[n];
        st_shared_f32(colv + 4 * i, cv);
      }
      // a BN = 256 warp owns one 128-column head: stage its norm weight
      const bool hn = FP4 && BN == 256 && ncol0 < p.hn_cols;
      if (hn) {  // as bf16 pairs: word i holds columns 2i, 2i + 1
        const uint32_t* wsrc = reinterpret_cast<const uint32_t*>(ncol0 < p.hn_q_cols ? p.hn_wq : p.hn_wk);
        for (int i = lane; i < C::kColsPerWarp / 2; i += 32)
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(hnv + 4 * i), "r"(__ldg(wsrc + i)) : "memory");
      }
      const int64_t row = (int64_t)m0 + q * 32 + lane;
      const bool row_ok = row < p.M;
      const int wblk = sm ? (n0 >> 7) : (ncol0 >> 7);  // weight-scale block of the (gate) columns
      const float a_row = (row_ok && p.a_gs) ? p.a_gs[p.a_gs_per_row ? row : 0] : 0.0f;
      const float alpha = (row_ok && p.a_gs) ? a_row * p.w_gs[p.w_gs_per_block ? wblk : 0] : 0.0f;
      const float alpha_u = sm ? a_row * p.w_gs[p.w_gs_per_block ? wblk + 1 : 0] : alpha;
      const __nv_bfloat16* gate_row =  // (the residual side tile carries the gate rows itself)
          (FP4 && p.gate && row_ok && !side_res) ? p.gate + (row / p.gate_rows) * p.ld_gate + ncol0 : nullptr;
      const __nv_bfloat16* res_row =
          (FP4 && p.residual && row_ok && !side_res) ? p.residual + row * p.ldr + ncol0 : nullptr;
#pragma unroll
      for (int j = 0; j < C::kColsPerWarp * 2; j += 128) {
        if (gate_row) prefetch_l2(reinterpret_cast<const uint8_t*>(gate_row) + j);
        if (res_row) prefetch_l2(reinterpret_cast<const uint8_t*>(res_row) + j);
      }
      if (gate_row) prefetch_l1(gate_row);  // the first 32-column chunk's segments into L1
      if (res_row) prefetch_l1(res_row);
      __syncwarp();
      if (!mbar_wait(acc_full, it & 1u, abort_flag, t0, p.status, 7, lim)) break;
      tc_fence_after();
      if (*abort_flag) break;
      uint32_t v[C::kChunks][32];
#pragma unroll
      for (int c = 0; c < C::kChunks; ++c)
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) +
                               (uint32_t)(sm ? (c < 2 ? 0 : 128) + half * 64 + (c & 1) * 32
                                             : half * C::kColsPerWarp + c * 32),
                           v[c]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {  // TMEM drained: the next tile's MMAs may start (the leader counts both CTAs)
        if (PAIR && !leader)
          mbar_arrive_cluster(acc_empty, 0);
        else
          mbar_arrive(acc_empty);
      }

      // row domain, one row per lane: y = bf16(alpha * acc + bias) (FP4), bf16(acc * col_scale / alpha)
      // (LoRA down-projection) or bf16(acc + bias) (plain bf16 linear: no column scale)
      const bool plain = !FP4 && !p.col_scale;
      const float inv_alpha = (FP4 || plain) ? 0.0f : (row_ok ? 1.0f / alpha : 0.0f);
      uint32_t y[C::kChunks][16];
#pragma unroll
      for (int c = 0; c < C::kChunks; ++c) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float4 cv = make_float4(0.f, 0.f, 0.f, 0.f);
          if constexpr (C::kColVec) {
            cv = ld_shared_f32x4(colv + 4 * (c * 32 + 4 * j));
          } else if constexpr (SIDE == 5) {  // four bias values, the same for every lane
            const int i0 = c * 32 + 4 * j;
            const int n = sm ? n0 + (i0 < 64 ? half * 64 + i0 : 128 + half * 64 + (i0 - 64)) : ncol0 + i0;
            const uint2 b2 = __ldg(reinterpret_cast<const uint2*>(p.bias + n));
            cv = make_float4(bf16_lo(b2.x), bf16_hi(b2.x), bf16_lo(b2.y), bf16_hi(b2.y));
          }
          if (FP4) {
            const float ac = (sm && c >= 2) ? alpha_u : alpha;
            const float2 al = make_float2(ac, ac);
            y[c][2 * j] = f2_bf2(fma_f2(al, make_float2(__uint_as_float(v[c][4 * j]), __uint_as_float(v[c][4 * j + 1])),
                                        make_float2(cv.x, cv.y)));
            y[c][2 * j + 1] = f2_bf2(fma_f2(
                al, make_float2(__uint_as_float(v[c][4 * j + 2]), __uint_as_float(v[c][4 * j + 3])),
                make_float2(cv.z, cv.w)));
          } else if (plain) {
            y[c][2 * j] = pack_bf16x2(__uint_as_float(v[c][4 * j]) + cv.x, __uint_as_float(v[c][4 * j + 1]) + cv.y);
            y[c][2 * j + 1] =
                pack_bf16x2(__uint_as_float(v[c][4 * j + 2]) + cv.z, __uint_as_float(v[c][4 * j + 3]) + cv.w);
          } else {
            y[c][2 * j] = pack_bf16x2(__uint_as_float(v[c][4 * j]) * (cv.x * inv_alpha),
                                      __uint_as_float(v[c][4 * j + 1]) * (cv.y * inv_alpha));
            y[c][2 * j + 1] = pack_bf16x2(__uint_as_float(v[c][4 * j + 2]) * (cv.z * inv_alpha),
                                          __uint_as_float(v[c][4 * j + 3]) * (cv.w * inv_alpha));
          }
        }
      }

      if constexpr (FP4 && BN == 256) {
        if (sm) {  // h = bf16(bf16(silu(g)) * u): chunks 0-1 gate, 2-3 the matching up columns
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int k = 0; k < 16; ++k) y[c][k] = silu_mul_bf2(y[c][k], y[c + 2][k]);
        }
      }
      // rotary tables of the row's position: their cache lines are pulled into L1 ahead of use
      // (no registers held), the first 64-column half's here, while the head norm runs
      const __nv_bfloat16* cos_row =
          (hn && p.rope_cos && !side_rope) ? p.rope_cos + (row % p.rope_S) * 128 : nullptr;
      const __nv_bfloat16* sin_row =
          (hn && p.rope_cos && !side_rope) ? p.rope_sin + (row % p.rope_S) * 128 : nullptr;
      if (cos_row) {
        prefetch_l1(cos_row);
        prefetch_l1(cos_row + 64);
        prefetch_l1(sin_row);
        prefetch_l1(sin_row + 64);
      }
      if (need_side && skey != cur) {
        if (!mbar_wait(side_full, sit & 1u, abort_flag, t0, p.status, 12, lim)) break;
        cur = skey;
      }
      const int srow = q * 32 + lane;  // the lane's row in the side tile
      if (hn) {
        // q_norm / k_norm: Qwen3RMSNorm over the row's 128 values of this head
        float se = 0.0f, so = 0.0f;  // even / odd columns' sums of squares
#pragma unroll
        for (int c = 0; c < C::kChunks; ++c)
#pragma unroll
          for (int k = 0; k < 16; ++k) sq_acc_bf2(y[c][k], se, so);
        // mean = sum / 128 as an exact power-of-two scaling (the same rounding as the division)
        const float rinv = __frsqrt_rn(__fadd_rn(__fmul_rn(__fadd_rn(se, so), 0.0078125f), p.hn_eps));
        const float2 r2 = make_float2(rinv, rinv);
#pragma unroll
        for (int c = 0; c < C::kChunks; ++c)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 w4 = ld_shared_v4(hnv + 4 * (c * 16 + 4 * j));
            const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)  // bf16(w * bf16(y * rinv))
              y[c][4 * j + i] = mul_bf2(f2_bf2(mul_f2(bf2_f2(y[c][4 * j + i]), r2)), ww[i]);
          }
        if (p.rope_cos) {
          // bf16(bf16(x * cos) + bf16(rotate_half(x) * sin)): column i < 64 pairs with i + 64
          const int64_t pos = row % p.rope_S;
          const uint4* cr = reinterpret_cast<const uint4*>(p.rope_cos + pos * 128);
          const uint4* sr = reinterpret_cast<const uint4*>(p.rope_sin + pos * 128);
          const uint32_t cb = side + srow * C::kSideRow, sb = cb + 128;  // staged cos / sin halves
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint4 c1, c2, s1, s2v;
              if (side_rope) {  // equal halves: columns i and i + 64 share their values
                c1 = c2 = ld_shared_v4(cb + (c * 4 + j) * 16);
                s1 = s2v = ld_shared_v4(sb + (c * 4 + j) * 16);
              } else {
                c1 = __ldg(cr + c * 4 + j);
                c2 = __ldg(cr + 8 + c * 4 + j);
                s1 = __ldg(sr + c * 4 + j);
                s2v = __ldg(sr + 8 + c * 4 + j);
              }
              const uint32_t cw1[4] = {c1.x, c1.y, c1.z, c1.w}, cw2[4] = {c2.x, c2.y, c2.z, c2.w};
              const uint32_t sw1[4] = {s1.x, s1.y, s1.z, s1.w}, sw2[4] = {s2v.x, s2v.y, s2v.z, s2v.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const uint32_t a = y[c][4 * j + i], b = y[c + 2][4 * j + i];
                // each product and the sum rounded to bf16 once (add_bf2: the exact sum of two
                // bf16 values rounded once equals the fp32 sum rounded to bf16)
                y[c][4 * j + i] = add_bf2(mul_bf2(a, cw1[i]), mul_bf2(b ^ 0x80008000u, sw1[i]));
                y[c + 2][4 * j + i] = add_bf2(mul_bf2(b, cw2[i]), mul_bf2(a, sw2[i]));
              }
            }
        }
      }
      if constexpr (SIDE == 2) {
        // out = bf16(residual + bf16(y * gate)) written over the lane's own residual chunks in
        // the side tile and stored from there, one 32-row x 64-column TMA box (the 128-byte
        // swizzle it was loaded with) per two chunks; the gate from its segments in the tile
        const bool gated = p.gate != nullptr;
        // the lane's gate row: the tile's first or second (a gate row spans >= 128 rows); the
        // loader stored the first row of the second one with the tile
        const int gnext = gated ? ld_shared_s32(side + C::kSideGate + 2 * BN * 2) : 0;
        const int gsel = (gated && (int)min(row, (int64_t)p.M - 1) >= gnext) ? 1 : 0;
        const uint32_t gb = side + C::kSideGate + gsel * (BN * 2) + half * (C::kColsPerWarp * 2);
#pragma unroll
        for (int bb = 0; bb < C::kChunks / 2; ++bb) {
          const int b = half * 2 + bb;  // 64-column box of the side tile
          const uint32_t rb = side + b * (kBM * 128) + srow * 128;
          // every shared-memory read of the box first (the in-place stores below would order
          // each read after the previous store), then the arithmetic and the stores
          uint4 rx[2][4], g4[2][4];
#pragma unroll
          for (int cc = 0; cc < 2; ++cc)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              rx[cc][j] = ld_shared_v4(rb + (((cc * 4 + j) ^ (srow & 7)) << 4));
              g4[cc][j] = gated ? ld_shared_v4(gb + (2 * bb + cc) * 64 + j * 16) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const int c = 2 * bb + cc;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t rw[4] = {rx[cc][j].x, rx[cc][j].y, rx[cc][j].z, rx[cc][j].w};
              const uint32_t gw[4] = {g4[cc][j].x, g4[cc][j].y, g4[cc][j].z, g4[cc][j].w};
              uint32_t o[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const uint32_t v = gated ? mul_bf2(y[c][4 * j + i], gw[i]) : y[c][4 * j + i];
                o[i] = add_bf2(rw[i], v);  // bf16(residual + y), as the fp32 sum rounded to bf16
              }
              st_shared_v4(rb + (((cc * 4 + j) ^ (srow & 7)) << 4), o[0], o[1], o[2], o[3]);
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {  // rows >= M are clipped by the tensor map
            const uint32_t src = side + b * (kBM * 128) + q * 32 * 128;
            if (p.out_evict_first)
              tma_store_2d_s_hint(&tmO, src, n0 + 64 * b, m0 + q * 32, out_policy);
            else
              tma_store_2d_s(&tmO, src, n0 + 64 * b, m0 + q * 32);
            bulk_commit();
          }
        }
        if (lane == 0) bulk_wait_read<0>();  // the stores have read the side tile
        __syncwarp();
      } else {
#pragma unroll
        for (int c = 0; c < C::kChunks; ++c) {
          if (sm && c >= 2) break;  // SwiGLU: two 32-column output chunks per warp
          if (c + 1 < C::kChunks) {  // the next chunk's gate / residual segments into L1
            if (gate_row) prefetch_l1(gate_row + (c + 1) * 32);
            if (res_row) prefetch_l1(res_row + (c + 1) * 32);
          }
          const int ncol = sm ? (n0 >> 1) + half * 64 + c * 32 : ncol0 + c * 32;
          // FP4 tiles never cross N (N % BN == 0); the bf16 GEMM's last tile can (rank < BN)
          if (!FP4 && ncol >= p.N) break;
          if (FP4) {
            if (gate_row) {  // y = bf16(y * gate), as the reference's eager `y * gate`
              uint4 gx[4];
              ld_global_row64(gate_row + c * 32, gx);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint32_t gw[4] = {gx[j].x, gx[j].y, gx[j].z, gx[j].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) y[c][4 * j + i] = mul_bf2(y[c][4 * j + i], gw[i]);
              }
            }
            if (res_row || side_res) {  // out = bf16(residual + y)
              uint4 rx[4];
              if (side_res) {  // box half * 2 + c / 2, 16-byte chunk k of the row at k ^ (row & 7)
                const uint32_t rb = side + (half * 2 + (c >> 1)) * (kBM * 128) + srow * 128;
#pragma unroll
                for (int j = 0; j < 4; ++j) rx[j] = ld_shared_v4(rb + ((((c & 1) * 4 + j) ^ (srow & 7)) << 4));
              } else {
                ld_global_row64(res_row + c * 32, rx);
              }
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint32_t rw[4] = {rx[j].x, rx[j].y, rx[j].z, rx[j].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) y[c][4 * j + i] = add_bf2(rw[i], y[c][4 * j + i]);
              }
            }
            // 32 rows x 32 columns, 64-byte swizzle (conflict-free), written by one TMA store;
            // two buffers per warp: wait only until the store before last has read its source
            const uint32_t buf = stg + (nstore & 1u) * 2048u;
            if (nstore >= 2) {
              if (lane == 0) bulk_wait_read<1>();
              __syncwarp();
            }
#pragma unroll
            for (int j = 0; j < 4; ++j)
              st_shared_v4(buf + stg_off(lane, j), y[c][4 * j], y[c][4 * j + 1], y[c][4 * j + 2], y[c][4 * j + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {  // rows >= M are clipped by the tensor map
              if (p.out_evict_first)
                tma_store_2d_s_hint(&tmO, buf, ncol, m0 + q * 32, out_policy);
              else
                tma_store_2d_s(&tmO, buf, ncol, m0 + q * 32);
              bulk_commit();
            }
            ++nstore;
          } else {
            // bf16 GEMM (LoRA down-projection, narrow outputs): transpose through shared
            // memory so each store instruction writes 8 rows x 64 contiguous bytes
#pragma unroll
            for (int j = 0; j < 4; ++j)
              st_shared_v4(stg + lane * kStgPitch + j * 16, y[c][4 * j], y[c][4 * j + 1], y[c][4 * j + 2],
                           y[c][4 * j + 3]);
            __syncwarp();
            const int trow = lane >> 2, tgr = lane & 3;
#pragma unroll
            for (int sp = 0; sp < 4; ++sp) {
              const int rl = trow + 8 * sp;
              const int64_t grow = (int64_t)m0 + q * 32 + rl;
              const uint4 o = ld_shared_v4(stg + rl * kStgPitch + tgr * 16);
              const int cc = ncol + tgr * 8;
              if (grow < p.M && cc < p.N) st_global_v4(p.out + grow * p.ldo + cc, o);
            }
            __syncwarp();
          }
        }
      }
      if (need_side && side_key(tile + t_step) != skey) {  // end of the run: release the side tile
        __syncwarp();
        if (lane == 0) mbar_arrive(side_empty);
        ++sit;
        cur = -1;
      }
    }
    if (FP4 && lane == 0) bulk_wait_all();  // the staging buffers stay valid until every store has read them
    __syncwarp();
  }

  tc_fence_before();
  if (PAIR)
    cluster_sync();  // no CTA of a pair leaves while the other may still touch its memory
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem, C::kTmemCols);
    else
      tmem_dealloc(tmem, C::kTmemCols);
  }
}

constexpr int kBandMBlocks = 8;

template <int BN, int STAGES, bool FP4, bool PAIR = false, int SIDE = 0>
int launch_gemm(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& la, const CUtensorMap& lb,
                const CUtensorMap& o, GemmParams p, cudaStream_t st, const CUtensorMap* sfa = nullptr,
                const CUtensorMap* sfb = nullptr, const CUtensorMap* res = nullptr) {
  using C = GemmCfg<BN, STAGES, FP4, PAIR, SIDE>;
  auto kern = gemm_kernel<BN, STAGES, FP4, PAIR, SIDE>;
  static std::atomic<uint64_t> attr_done{0};
  if (device_pending(attr_done)) {
    // the warpgroups' register split adds up to the launch's registers; with any other count
    // per thread at launch the epilogue's setmaxnreg.inc would never return
    cudaFuncAttributes fa;
    DEMON_CUDA(cudaFuncGetAttributes(&fa, kern));
    if (fa.numRegs != kGemmLaunchRegs) {
      set_error("gemm: kernel built with %d registers per thread, the register split needs %d", fa.numRegs,
                kGemmLaunchRegs);
      return DEMON_ERR_CUDA;
    }
    DEMON_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    mark_device_done(attr_done);
  }
  int dev = 0, sms = 148;
  DEMON_CUDA(cudaGetDevice(&dev));
  DEMON_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  constexpr int tile_m = PAIR ? 2 * kBM : kBM;
  p.m_tiles = (p.M + tile_m - 1) / tile_m;
  p.n_tiles = (p.N + BN - 1) / BN;
  const int tiles = p.m_tiles * p.n_tiles;
  // A operand bytes beyond ~24 MB do not survive in L2 next to the streaming output, so
  // large-M launches sweep N in bands of 8 m-blocks; smaller ones keep m-fastest order
  const double a_bytes = (double)p.M * p.K * (FP4 ? 0.5625 : 2.0);
  p.m_group = (a_bytes > 24e6) ? std::min(p.m_tiles, kBandMBlocks) : p.m_tiles;
  if (SIDE == 1) {
    // each pair sweeps N over its own m-blocks (contiguous tiles, n fastest): the rotary
    // tables of an m-block are loaded once for all its head tiles; the pairs' A blocks
    // (256 KB each) stay in L2 while they are swept
    const int pairs = std::min(tiles, sms / 2);
    p.m_group = 1;
    p.tile_chunk = (tiles + pairs - 1) / pairs;
  }
  CUtensorMap z;
  memset(&z, 0, sizeof z);
  if (!PAIR) {
    const dim3 grid((unsigned)std::min(tiles, sms));
    kern<<<grid, kThreads, C::kSmem, st>>>(a, b, la, lb, o, z, z, z, p);
    DEMON_CUDA(cudaGetLastError());
    return DEMON_OK;
  }
  // persistent CTA pairs: one pair per two SMs, clusters of 2
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * std::min(tiles, sms / 2)));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // griddepcontrol in the kernel
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  DEMON_CUDA(cudaLaunchKernelEx(&cfg, kern, a, b, la, lb, o, sfa ? *sfa : z, sfb ? *sfb : z, res ? *res : z, p));
  return DEMON_OK;
}

}  // namespace demon

namespace demon {
// CTA-pair tiles are the default for N % 256 == 0; DEMON_GEMM_PAIR=0 selects the one-CTA
// kernel (kept for comparison and as the N % 256 != 0 path).
static bool side_stage_enabled() {
  static const bool on = [] {
    const char* e = getenv("DEMON_GEMM_SIDE");
    return !(e && e[0] == '0');
  }();
  return on;
}
static bool pair_gemm_enabled() {
  static const bool on = [] {
    const char* e = getenv("DEMON_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}
}  // namespace demon

using namespace demon;

#define DEMON_RC(x)             \
  do {                          \
    int _rc = (x);              \
    if (_rc != DEMON_OK) return _rc; \
  } while (0)

namespace demon {
int gemm_check(const DemonGemmArgs* a) {
  DEMON_CHECK_ARG(a != nullptr, "gemm: null args");
  const int64_t M = a->M, N = a->N, K = a->K;
  DEMON_CHECK_ARG(M >= 0 && N > 0 && K > 0, "gemm: bad shape M=%lld N=%lld K=%lld", (long long)M, (long long)N,
                  (long long)K);
  DEMON_CHECK_ARG(K % 256 == 0, "gemm: K must be a multiple of 256 (K=%lld)", (long long)K);
  DEMON_CHECK_ARG(N % 128 == 0, "gemm: N must be a multiple of 128 (N=%lld)", (long long)N);
  DEMON_CHECK_ARG(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "gemm: dimension too large");
  DEMON_CHECK_ARG(a->a_codes && a->a_sf && a->a_gs && a->w_codes && a->w_sf && a->w_gs && a->out,
                  "gemm: null operand");
  DEMON_CHECK_ARG(((uintptr_t)a->a_codes & 15) == 0 && ((uintptr_t)a->w_codes & 15) == 0,
                  "gemm: code buffers must be 16-byte aligned");
  DEMON_CHECK_ARG(a->ldo >= (a->silu_mul ? N / 2 : N) && a->ldo % 8 == 0 && ((uintptr_t)a->out & 15) == 0,
                  "gemm: out needs ldo >= N (N / 2 with silu_mul), ldo %% 8 == 0, 16-byte alignment");
  DEMON_CHECK_ARG(!a->residual || (a->ldr >= N && a->ldr % 8 == 0 && ((uintptr_t)a->residual & 15) == 0),
                  "gemm: residual needs ldr >= N, ldr %% 8 == 0, 16-byte alignment");
  DEMON_CHECK_ARG(!a->bias || ((uintptr_t)a->bias & 15) == 0, "gemm: bias must be 16-byte aligned");
  DEMON_CHECK_ARG(!a->gate || (a->gate_rows > 0 && a->ld_gate >= N && a->ld_gate % 8 == 0 &&
                               ((uintptr_t)a->gate & 15) == 0),
                  "gemm: gate needs gate_rows > 0, ld_gate >= N, ld_gate %% 8 == 0, 16-byte alignment");
  DEMON_CHECK_ARG(((uintptr_t)a->a_sf & 15) == 0 && ((uintptr_t)a->w_sf & 15) == 0,
                  "gemm: scale buffers must be 16-byte aligned");
  const bool lora = a->lora_xa != nullptr;
  DEMON_CHECK_ARG(!lora || (a->lora_b && a->lora_rank > 0 && a->lora_rank % 16 == 0 && a->lora_rank <= 128),
                  "gemm: LoRA needs lora_b and rank %% 16 == 0, 0 < rank <= 128 (rank=%lld)",
                  (long long)a->lora_rank);
  DEMON_CHECK_ARG(!lora || (((uintptr_t)a->lora_xa & 15) == 0 && ((uintptr_t)a->lora_b & 15) == 0),
                  "gemm: LoRA operands must be 16-byte aligned");
  DEMON_CHECK_ARG(!(lora && a->w_gs_per_block), "gemm: hot LoRA needs a single weight scale (w_gs_per_block = 0)");
  if (a->hn_cols > 0) {
    DEMON_CHECK_ARG(N % 256 == 0 && a->hn_cols % 128 == 0 && a->hn_cols <= N && a->hn_q_cols >= 0 &&
                        a->hn_q_cols % 128 == 0 && a->hn_q_cols <= a->hn_cols,
                    "gemm: head norm needs N %% 256 == 0 and hn_q_cols <= hn_cols <= N, both multiples of 128");
    DEMON_CHECK_ARG(!a->gate && !a->residual, "gemm: head norm excludes gate / residual");
    DEMON_CHECK_ARG((a->hn_q_cols == 0 || a->hn_wq) && (a->hn_q_cols == a->hn_cols || a->hn_wk),
                    "gemm: head norm weight missing");
    DEMON_CHECK_ARG(!a->rope_cos || (a->rope_sin && a->rope_S > 0 && ((uintptr_t)a->rope_cos & 15) == 0 &&
                                     ((uintptr_t)a->rope_sin & 15) == 0),
                    "gemm: rotary tables need rope_sin, rope_S > 0 and 16-byte alignment");
  }
  const bool silu = a->silu_mul != 0;
  DEMON_CHECK_ARG(!silu || (N % 256 == 0 && !lora && a->hn_cols == 0 && !a->gate && !a->residual),
                  "gemm: the SwiGLU epilogue needs N %% 256 == 0 and excludes LoRA, head norm, gate, residual");
  return DEMON_OK;
}

namespace {
// demon_test_arm_gemm_stall: wait limit (ns) for the next NVFP4 GEMM launch of this thread
thread_local int64_t t_stall_wait_ns = 0;
}  // namespace
}  // namespace demon

extern "C" int demon_test_arm_gemm_stall(int64_t wait_ns) {
  DEMON_CHECK_ARG(wait_ns == 0 || (wait_ns >= 100000 && wait_ns <= 1000000000),
                  "test_arm_gemm_stall: wait_ns must be 0 or in [1e5, 1e9] (%lld)", (long long)wait_ns);
  demon::t_stall_wait_ns = wait_ns;
  return DEMON_OK;
}

extern "C" int demon_nvfp4_gemm(const DemonGemmArgs* a, void* stream) {
  DEMON_API_BEGIN();
  const int rc0 = gemm_check(a);
  if (rc0 != DEMON_OK) return rc0;
  const int64_t M = a->M, N = a->N, K = a->K;
  const bool lora = a->lora_xa != nullptr;
  const bool silu = a->silu_mul != 0;
  const int64_t n_out = silu ? N / 2 : N;
  if (M == 0) return DEMON_OK;

  const bool bn256 = (N % 256 == 0);
  const uint32_t BN = bn256 ? 256 : 128;
  CUtensorMap ta, tb, tla, tlb;
  memset(&tla, 0, sizeof tla);
  memset(&tlb, 0, sizeof tlb);
  DEMON_RC(make_tmap_2d(&ta, a->a_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)K / 2, (uint64_t)M,
                        (uint64_t)K / 2, 128, 128));
  // N % 256 == 0: 256 x 256 tiles on CTA pairs (each CTA loads half of the B tile)
  const bool pair = bn256 && pair_gemm_enabled();
  DEMON_RC(make_tmap_2d(&tb, a->w_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)K / 2, (uint64_t)N,
                        (uint64_t)K / 2, 128, pair ? BN / 2 : BN));
  // scale buffers as rows of 256 bytes: one 2 KB box is one stage's 128-row scale chunk run
  CUtensorMap tsfa, tsfb;
  memset(&tsfa, 0, sizeof tsfa);
  memset(&tsfb, 0, sizeof tsfb);
  if (pair) {
    DEMON_RC(make_tmap_2d(&tsfa, a->a_sf, CU_TENSOR_MAP_DATA_TYPE_UINT8, 256,
                          (uint64_t)(((M + 127) / 128) * K / 32), 256, 256, 8, CU_TENSOR_MAP_SWIZZLE_NONE));
    DEMON_RC(make_tmap_2d(&tsfb, a->w_sf, CU_TENSOR_MAP_DATA_TYPE_UINT8, 256,
                          (uint64_t)(((N + 127) / 128) * K / 32), 256, 256, 8, CU_TENSOR_MAP_SWIZZLE_NONE));
  }
  // output: 32 x 32 bf16 store boxes (64-byte rows, 64-byte swizzle); rows past M are clipped
  CUtensorMap to;
  DEMON_RC(make_tmap_2d(&to, a->out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)n_out, (uint64_t)M,
                        (uint64_t)a->ldo * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B));
  if (lora) {
    const uint64_t r = (uint64_t)a->lora_rank;
    DEMON_RC(make_tmap_2d(&tla, a->lora_xa, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, r, (uint64_t)M, r * 2, 64, 128));
    DEMON_RC(make_tmap_2d(&tlb, a->lora_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, r, (uint64_t)N, r * 2, 64,
                          pair ? BN / 2 : BN));
  }
  GemmParams p{};
  p.a_sf = a->a_sf;
  p.w_sf = a->w_sf;
  p.a_gs = a->a_gs;
  p.w_gs = a->w_gs;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(a->bias);
  p.gate = reinterpret_cast<const __nv_bfloat16*>(a->gate);
  p.residual = reinterpret_cast<const __nv_bfloat16*>(a->residual);
  p.out = reinterpret_cast<__nv_bfloat16*>(a->out);
  p.ldo = a->ldo;
  p.ldr = a->ldr;
  p.status = status_word();
  p.gate_rows = a->gate_rows > 0 ? a->gate_rows : 1;
  p.ld_gate = a->ld_gate;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.a_gs_per_row = a->a_gs_per_row;
  p.w_gs_per_block = a->w_gs_per_block;
  p.hn_cols = (int)a->hn_cols;
  p.hn_q_cols = (int)a->hn_q_cols;
  p.rope_S = a->rope_S > 0 ? a->rope_S : 1;
  p.hn_wq = reinterpret_cast<const __nv_bfloat16*>(a->hn_wq);
  p.hn_wk = reinterpret_cast<const __nv_bfloat16*>(a->hn_wk);
  p.rope_cos = reinterpret_cast<const __nv_bfloat16*>(a->rope_cos);
  p.rope_sin = reinterpret_cast<const __nv_bfloat16*>(a->rope_sin);
  p.hn_eps = a->hn_eps;
  p.silu_mul = silu ? 1 : 0;
  p.lora_rank = lora ? (int)a->lora_rank : 0;
  // an output larger than L2 cannot stay there for the next kernel: stream it out first, so
  // that it does not evict the operand tiles the other CTAs are still reading (~5 % at
  // M = 96000, N = 12288)
  p.out_evict_first = (double)M * (double)n_out * 2.0 > 100e6 ? 1 : 0;
  if (t_stall_wait_ns > 0) {  // armed bounded-wait test: one launch only
    p.withhold = 1;
    p.wait_ns = (uint64_t)t_stall_wait_ns;
    t_stall_wait_ns = 0;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // A side tile when the epilogue would otherwise read per-row operands one row per lane
  // (gemm_check: never both, never with SwiGLU; residual rows 16-byte aligned): the rotary
  // tables of the head-norm + RoPE epilogue when their halves are equal (rope_half: 34 KB, four
  // stages; full tables are read directly), or the residual, which the output overwrites and
  // is stored from (no staging buffers: four stages, 64 x 32 store boxes), with the gate rows
  // when each spans at least a tile's 128 rows
  const bool side_rope = a->rope_cos && a->hn_cols > 0 && a->rope_half;
  const bool side_res = a->residual != nullptr && !a->bias && (!a->gate || a->gate_rows >= 128);
  if (pair && side_stage_enabled() && side_rope)
    return launch_gemm<256, 4, true, true, 1>(ta, tb, tla, tlb, to, p, st, &tsfa, &tsfb);
  if (pair && side_stage_enabled() && side_res) {
    CUtensorMap tr, to2;
    DEMON_RC(make_tmap_2d(&tr, a->residual, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)N, (uint64_t)M,
                          (uint64_t)a->ldr * 2, 64, 128));
    DEMON_RC(make_tmap_2d(&to2, a->out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)n_out, (uint64_t)M,
                          (uint64_t)a->ldo * 2, 64, 32));
    return launch_gemm<256, 4, true, true, 2>(ta, tb, tla, tlb, to2, p, st, &tsfa, &tsfb, &tr);
  }
  // no bias (and no side tile above): no per-column vector, and its shared memory buys a fifth
  // stage (the SwiGLU gate/up GEMM: 1190 -> 985 us at M = 96,000)
  if (pair && !a->bias)
    return launch_gemm<256, 5, true, true, 3>(ta, tb, tla, tlb, to, p, st, &tsfa, &tsfb);
  if (pair && !a->residual)  // a bias but no residual (config 1's linear): the bias from global memory
    return launch_gemm<256, 5, true, true, 5>(ta, tb, tla, tlb, to, p, st, &tsfa, &tsfb);
  if (pair) return launch_gemm<256, 4, true, true>(ta, tb, tla, tlb, to, p, st, &tsfa, &tsfb);
  if (bn256) return launch_gemm<256, 3, true>(ta, tb, tla, tlb, to, p, st);
  return launch_gemm<128, 5, true>(ta, tb, tla, tlb, to, p, st);
}

extern "C" int demon_lora_down(const void* x, int64_t M, int64_t K, int64_t ldx, const void* lora_a, int64_t rank,
                               const float* col_scale, const float* a_gs, int a_gs_per_row, const float* w_gs,
                               void* xa, void* stream) {
  DEMON_API_BEGIN();
  DEMON_CHECK_ARG(M >= 0 && K > 0 && K % 64 == 0, "lora_down: need K %% 64 == 0 (K=%lld)", (long long)K);
  DEMON_CHECK_ARG(rank > 0 && rank % 16 == 0 && rank <= 128, "lora_down: rank %% 16 == 0, rank <= 128 (%lld)",
                  (long long)rank);
  DEMON_CHECK_ARG(ldx >= K && ldx % 8 == 0, "lora_down: ldx must be >= K and a multiple of 8");
  DEMON_CHECK_ARG(x && lora_a && col_scale && a_gs && w_gs && xa, "lora_down: null pointer");
  DEMON_CHECK_ARG(((uintptr_t)xa & 15) == 0, "lora_down: xa must be 16-byte aligned");
  if (M == 0) return DEMON_OK;
  CUtensorMap ta, tb, tz;
  memset(&tz, 0, sizeof tz);
  DEMON_RC(make_tmap_2d(&ta, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)K, (uint64_t)M, (uint64_t)ldx * 2, 64,
                        128));
  GemmParams p{};
  p.a_gs = a_gs;
  p.w_gs = w_gs;
  p.col_scale = col_scale;
  p.out = reinterpret_cast<__nv_bfloat16*>(xa);
  p.ldo = rank;
  p.status = status_word();
  p.M = (int)M;
  p.N = (int)rank;
  p.K = (int)K;
  p.a_gs_per_row = a_gs_per_row;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (rank <= 64) {
    DEMON_RC(make_tmap_2d(&tb, lora_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)K, (uint64_t)rank,
                          (uint64_t)K * 2, 64, 64));
    return launch_gemm<64, 6, false>(ta, tb, tz, tz, tz, p, st);
  }
  DEMON_RC(make_tmap_2d(&tb, lora_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)K, (uint64_t)rank,
                        (uint64_t)K * 2, 64, 128));
  return launch_gemm<128, 6, false>(ta, tb, tz, tz, tz, p, st);
}

extern "C" int demon_bf16_linear(const void* x, int64_t M, int64_t K, int64_t ldx, const void* w, int64_t N,
                                 const void* bias, void* out, int64_t ldo, void* stream) {
  DEMON_API_BEGIN();
  DEMON_CHECK_ARG(M >= 0 && K > 0 && K % 64 == 0 && N > 0 && N % 64 == 0,
                  "bf16_linear: need K %% 64 == 0, N %% 64 == 0 (K=%lld N=%lld)", (long long)K, (long long)N);
  DEMON_CHECK_ARG(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "bf16_linear: dimension too large");
  DEMON_CHECK_ARG(ldx >= K && ldx % 8 == 0 && ldo >= N && ldo % 8 == 0,
                  "bf16_linear: ldx >= K, ldo >= N, both multiples of 8");
  DEMON_CHECK_ARG(x && w && out, "bf16_linear: null pointer");
  DEMON_CHECK_ARG(((uintptr_t)out & 15) == 0 && (!bias || ((uintptr_t)bias & 15) == 0),
                  "bf16_linear: out and bias must be 16-byte aligned");
  if (M == 0) return DEMON_OK;
  CUtensorMap ta, tb, tz;
  memset(&tz, 0, sizeof tz);
  DEMON_RC(make_tmap_2d(&ta, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)K, (uint64_t)M, (uint64_t)ldx * 2, 64,
                        128));
  GemmParams p{};
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.status = status_word();
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (N % 128 != 0) {
    DEMON_RC(make_tmap_2d(&tb, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)K, (uint64_t)N, (uint64_t)K * 2, 64,
                          64));
    return launch_gemm<64, 6, false>(ta, tb, tz, tz, tz, p, st);
  }
  DEMON_RC(make_tmap_2d(&tb, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)K, (uint64_t)N, (uint64_t)K * 2, 64,
                        128));
  return launch_gemm<128, 6, false>(ta, tb, tz, tz, tz, p, st);
}
