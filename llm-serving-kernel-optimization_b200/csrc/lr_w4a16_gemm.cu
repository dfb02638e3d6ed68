// lr_w4a16_gemm.cu -- grouped W4A16 expert GEMM on tcgen05 (sm_100a).
//
// Tile: token rows of one expert (the UMMA M operand, K-major, TMA loaded) x
// WN dequantized weight columns (the UMMA N operand, MN-major, written by the
// dequant warps).  For SwiGLU the WN columns are WN/2 gate and the same WN/2 up
// features, so one accumulator row holds both halves of every output it needs.
// Accumulators (TMEM lane = token row, one fp32 column per weight column) are
// double buffered so the epilogue of one tile overlaps the main loop of the next.
//
// Two tile shapes share the kernel (MT = number of 128-row M sub-tiles):
//   MT = 1, WN = 256: short expert segments (decode).  Each tcgen05.mma is
//     issued by one thread at a roughly fixed cost, so 256 weight columns
//     (2 KB of INT4 per 16-deep step) stand behind every instruction; only
//     TOKROWS (32, 64 or 128) token rows are loaded per stage and the rest of
//     the 128 M rows are left unused.
//   MT = 2, WN = 128: long segments (prefill).  256 token rows share each
//     dequantized weight column, halving the dequant work (the CUDA-core side
//     of the pipeline) per tensor-core FLOP.
//
// Warp roles (576 threads, one CTA per SM, persistent over tiles):
//   warps 0-7   epilogue, two groups of four (warp w reads TMEM lanes 32*(w%4)..);
//               MT = 2: group g drains M sub-tile g; MT = 1: the groups take
//               alternate 16-column chunks.  tcgen05.ld -> activation -> fp16 ->
//               16-byte stores of the token row
//   warps 8-15  dequant, in DGROUPS groups that take alternate k-steps: packed
//               int32 words (TMA-staged) + per-group scale / zero (read from
//               global memory) -> fp16(scale * (q - zero)), written into the
//               128-byte-swizzled MN-major operand buffer of their k-step
//   warp 16     token producer: TMA loads of the token box into the token ring,
//               whose stages the MMA releases (tcgen05.commit)
//   warp 17     weight producer: TMA loads of the packed weight box(es) into the
//               weight ring, whose stages the dequant warps release as soon as
//               they have read the words, so weights run ahead of the MMA
//   warp 18     TMEM allocation + single-thread tcgen05.mma issue
//
// Every mbarrier wait is bounded in time; a wait that runs out raises a
// shared abort flag and LR_DEVERR_PIPE_TIMEOUT so all roles drain and exit.
#include <cstring>

#include "lr_w4a16.cuh"

namespace lr {

constexpr int kEpiWarps = 8;
constexpr int kDeqWarps = 8;
constexpr int kProdWarp = kEpiWarps + kDeqWarps;  // token ring
constexpr int kWProdWarp = kProdWarp + 1;         // packed-weight ring
constexpr int kMmaWarp = kWProdWarp + 1;
constexpr int kGemmThreads = (kMmaWarp + 1) * 32;

// Tile shape: MT sub-tiles of 128 M rows (TOKROWS loaded per sub-tile) x WN
// weight columns; STAGES TMA stages (tokens + packed weights), DSTAGES
// dequantized-operand buffers and DGROUPS dequant warp groups.  The
// accumulator takes MT * WN TMEM columns; it is double buffered when two fit
// in the 512 columns of an SM, otherwise the epilogue of a tile and the main
// loop of the next one take turns.
template <int TOKROWS_, int MT_, int WN_, int STAGES_, int DSTAGES_, int DGROUPS_>
struct GemmShape {
  static constexpr int TOKROWS = TOKROWS_, MT = MT_, WN = WN_, STAGES = STAGES_,
                       DSTAGES = DSTAGES_, DGROUPS = DGROUPS_;
  static constexpr int ACC = MT * WN;                  // TMEM columns per accumulator
  static constexpr int NACC = 2 * ACC <= 512 ? 2 : 1;  // accumulator buffers
  static constexpr int WJ = WN / 8;                    // packed words per weight row
  static constexpr int ROWS = MT * TOKROWS;            // token rows per tile
  // UMMA M: 64 when a single sub-tile loads at most 64 rows.  An M = 64
  // accumulator keeps row i in TMEM lane 32*(i/16) + i%16 (16 lanes of each
  // warp's quarter).
  static constexpr int UM = (MT == 1 && TOKROWS <= 64) ? 64 : 128;
  static constexpr int RQ = UM / 4;  // accumulator rows per TMEM lane quarter
  static constexpr int kAStage = ROWS * kBK * 2;       // token box bytes
  static constexpr int kWStage = kBK * WN / 2;         // packed weight bytes per stage
  static constexpr int kBBuf = WN * kBK * 2;           // dequantized operand buffer
  static constexpr int offA = 0;
  static constexpr int offB = offA + STAGES * kAStage;
  static constexpr int offW = offB + DSTAGES * kBBuf;
  static constexpr int offBar = offW + STAGES * kWStage;
  static constexpr int kNumBars = 4 * STAGES + DSTAGES + 4 + 1;
  static constexpr int offMisc = offBar + kNumBars * 8;
  static constexpr int offTab = offMisc + 8 * 4;
  static constexpr int kTabBytes = (kMaxGemmExperts * 4 + 1) * 4;
  static constexpr int kTotal = offTab + kTabBytes + 1024;  // + base alignment slack
  static_assert(offB % 1024 == 0 && offW % 1024 == 0, "operand alignment");
  static_assert(MT == 1 || TOKROWS == 128, "stacked M sub-tiles are full");
  static_assert(ROWS <= 256, "TMA box height");
  static_assert(kDeqWarps % DGROUPS == 0 && DGROUPS <= DSTAGES, "dequant groups");
  static_assert(kTotal <= 227 * 1024, "shared memory budget");
  static_assert(NACC * ACC <= 512 && WN % 64 == 0 && WN <= 256, "TMEM accumulators");
};

using ShapeR32 = GemmShape<32, 1, 256, 7, 4, 4>;
using ShapeR64 = GemmShape<64, 1, 256, 5, 4, 4>;
using ShapeR128 = GemmShape<128, 1, 256, 6, 2, 2>;
using ShapeR256 = GemmShape<128, 2, 128, 4, 4, 2>;   // double-buffered accumulator
using ShapeR256W = GemmShape<128, 2, 256, 3, 3, 2>;  // 256x256 tile, one accumulator
// K at and above which the 256x256 tile pays: its epilogue is not overlapped
// with the next tile's main loop, so it needs enough k-steps to amortise.
constexpr int kWideTileMinK = 4096;

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <class S, int MODE>
__global__ void __launch_bounds__(kGemmThreads, 1)
    w4a16_grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                              const ExpertEntry* __restrict__ table, int E, int mat, int K, int N,
                              const int32_t* __restrict__ seg_start,
                              const int32_t* __restrict__ seg_len, int max_rows, int R,
                              __half* __restrict__ C, int32_t* err, int n_fastest) {
  constexpr int STAGES = S::STAGES, DSTAGES = S::DSTAGES, DGROUPS = S::DGROUPS;
  constexpr int MT = S::MT, WN = S::WN, WJ = S::WJ, ROWS = S::ROWS;
  constexpr bool kGLU = MODE == LR_FFN_MODE_SWIGLU;
  constexpr int BO = kGLU ? WN / 2 : WN;  // output features per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sA = smem + S::offA;
  uint8_t* sB = smem + S::offB;
  uint32_t* sW = reinterpret_cast<uint32_t*>(smem + S::offW);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::offBar);  // token stage loaded
  uint64_t* empty = full + STAGES;    // token stage released by the MMA
  uint64_t* wfull = empty + STAGES;   // packed-weight stage loaded
  uint64_t* wempty = wfull + STAGES;  // packed-weight stage read by its dequant group
  uint64_t* dfull = wempty + STAGES;
  uint64_t* tfull = dfull + DSTAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* fin = tempty + 2;
  int* misc = reinterpret_cast<int*>(smem + S::offMisc);
  volatile int* s_abort = misc;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(misc + 1);
  int* s_tbase = reinterpret_cast<int*>(smem + S::offTab);  // E+1
  int* s_start = s_tbase + E + 1;                            // E
  int* s_len = s_start + E;                                  // E
  int* s_mt = s_len + E;                                     // E

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (N + BO - 1) / BO;
  const int KB = K / kBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      mbar_init(&wfull[i], 1);
      mbar_init(&wempty[i], kDeqWarps / DGROUPS);
    }
    for (int i = 0; i < DSTAGES; ++i) mbar_init(&dfull[i], kDeqWarps / DGROUPS);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kEpiWarps * 32);
    }
    mbar_init(fin, 1);
    *s_abort = 0;
    fence_mbarrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(s_tmem, S::NACC * S::ACC);
    tmem_relinquish();
  }
  if (warp == kProdWarp) {
    if (lane == 0) tma_prefetch_desc(&tmap_a);
    build_tile_table(seg_start, seg_len, E, R, max_rows, ROWS, n_tiles, s_tbase, s_start, s_len,
                     s_mt, err);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int total = s_tbase[E];

  // tile -> (expert, token tile, feature tile); token tiles vary fastest
  auto decode = [&](int tile, int& e, int& mt, int& nt) {
    decode_tile(s_tbase, s_mt, E, tile, e, mt, nt, n_fastest != 0, n_tiles);
  };

  if (warp == kProdWarp) {
    // ------------------------------------------------------------ token producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
        int e, mt, nt;
        decode(tile, e, mt, nt);
        const int row0 = s_start[e] + mt * ROWS;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!wait_any(&empty[s], ph ^ 1, s_abort, err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], uint32_t(S::kAStage));
          tma_load_2d(sA + s * S::kAStage, &tmap_a, &full[s], kb * kBK, row0);
        }
      }
      if (ok) {
        // Producer tail: wait until the MMA has released every stage.  The
        // releases are tcgen05.commit arrivals that complete asynchronously;
        // leaving before they land would let them hit the barriers of the next
        // CTA placed on this SM.  (The dequant buffers are released by the same
        // arrivals.)
        for (int i = 0; i < STAGES; ++i, ++it) {
          if (!wait_any(&empty[it % STAGES], ((it / STAGES) & 1) ^ 1, s_abort, err)) break;
        }
      } else {
        // let in-flight copies land before the CTA exits
        const int first = it - STAGES < 0 ? 0 : it - STAGES;
        for (int i = first; i < it; ++i) wait_drain(&full[i % STAGES], (i / STAGES) & 1);
      }
    }
  } else if (warp == kWProdWarp) {
    // ------------------------------------------------------------ weight producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
        int e, mt, nt;
        decode(tile, e, mt, nt);
        const ExpertEntry* ent = table + e;
        const int n0 = nt * BO;
        // PLAIN / SILU: one box of WJ words; SwiGLU: WJ/2 gate + WJ/2 up words
        const CUtensorMap* wmap0;
        if (kGLU) wmap0 = WN == 256 ? &ent->qw16[0] : &ent->qw8[0];
        else wmap0 = WN == 256 ? &ent->qw32[mat] : &ent->qw16[mat];
        const CUtensorMap* wmap1 = WN == 256 ? &ent->qw16[1] : &ent->qw8[1];
        // descriptors were written to global memory by a copy before the launch
        tensormap_acquire(wmap0);
        if (kGLU) tensormap_acquire(wmap1);
        // only the packed weight box(es) travel by TMA; the small per-group
        // scale / zero rows are read by the dequant warps
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!wait_any(&wempty[s], ph ^ 1, s_abort, err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&wfull[s], uint32_t(S::kWStage));
          uint32_t* w = sW + s * (S::kWStage / 4);
          tma_load_2d(w, wmap0, &wfull[s], n0 / 8, kb * kBK);
          if (kGLU) tma_load_2d(w + S::kWStage / 8, wmap1, &wfull[s], n0 / 8, kb * kBK);
        }
      }
      // Weight stages are released by ordinary arrivals of the dequant warps,
      // so nothing arrives here after the loop; the last copies (which the
      // dequant warps may not wait for after an abort) must land before the
      // CTA exits.
      (void)ok;
      const int first = it - STAGES < 0 ? 0 : it - STAGES;
      for (int i = first; i < it; ++i) wait_drain(&wfull[i % STAGES], (i / STAGES) & 1);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(S::UM, WN, 0, 1);
      int it = 0, lt = 0;
      bool ok = true;
      // Readiness of k-step `it` observed ahead of time: the barriers of the
      // next k-step are tested (non-blocking) before this k-step's MMAs are
      // issued; a blocking wait is needed only when the test came back false.
      bool pre_full = false, pre_dfull = false;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x, ++lt) {
        const int acc = S::NACC == 2 ? (lt & 1) : 0;
        const uint32_t aph = S::NACC == 2 ? (lt >> 1) & 1 : lt & 1;
        if (!wait_any(&tempty[acc], aph ^ 1, s_abort, err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * S::ACC);
        // stacked M sub-tiles: a tile of at most 128 token rows (small experts,
        // segment tails) skips the second sub-tile's MMAs; those accumulator
        // rows are never read (the epilogue clips to the tile's rows)
        int m_used = MT;
        if (MT == 2) {
          int e, mt, nt;
          decode(tile, e, mt, nt);
          if (s_len[e] - mt * ROWS <= 128) m_used = 1;
        }
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          const int q = it % DSTAGES;
          const uint32_t qph = (it / DSTAGES) & 1;
          if ((!pre_full && !wait_any(&full[s], ph, s_abort, err)) ||
              (!pre_dfull && !wait_any(&dfull[q], qph, s_abort, err))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int it2 = it + 1;  // next k-step of this CTA's stream (maybe the next tile's)
          const bool more = kb + 1 < KB || tile + int(gridDim.x) < total;
          const bool nf = more && mbar_test_wait(&full[it2 % STAGES], (it2 / STAGES) & 1);
          const bool nd = more && mbar_test_wait(&dfull[it2 % DSTAGES], (it2 / DSTAGES) & 1);
          const uint32_t aaddr = smem_u32(sA + s * S::kAStage);
          const uint32_t baddr = smem_u32(sB + q * S::kBBuf);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t bdesc = umma_smem_desc(baddr + kk * 2048, 8192, 1024, 2);
#pragma unroll
            for (int m = 0; m < MT; ++m) {
              if (m >= m_used) break;
              // M sub-tile m: token rows 128m.. (16 KB into the stage), TMEM columns WN*m..
              const uint64_t adesc = umma_smem_desc(aaddr + m * 16384 + kk * 32, 16, 1024, 2);
              umma_f16_ss(d_tmem + uint32_t(m * WN), adesc, bdesc, idesc,
                          (kb | kk) != 0 ? 1u : 0u);
            }
          }
          // one release for both the token stage and the dequantized buffer
          umma_commit(&empty[s]);
          pre_full = nf;
          pre_dfull = nd;
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      if (!ok) {
        umma_commit(fin);
        wait_drain(fin, 0);
      }
    }
  } else if (warp >= kEpiWarps) {
    // ------------------------------------------------------------ dequant
    // DGROUPS groups of kWg warps; group g converts the k-steps it with
    // it % DGROUPS == g into operand buffer it % DSTAGES, so several k-steps
    // (each a dependent load -> convert -> store -> fence chain) can be in
    // flight at once.  A buffer is free again once the MMA of the k-step that
    // used it before (it - DSTAGES) completed, i.e. once that k-step's stage was
    // released.
    constexpr int kWg = kDeqWarps / DGROUPS;          // warps per group
    constexpr int kGT = 32 * kWg;                     // threads per group
    constexpr int kWords = (S::kWStage / 4) / kGT;    // packed words per thread per k-step
    constexpr int kRowStep = kGT / WJ;                // rows between a thread's words
    static_assert(kWords * kRowStep == kBK, "dequant thread mapping");
    const int dtid = threadIdx.x - kEpiWarps * 32;
    const int dgrp = dtid / kGT;
    const int gt = dtid % kGT;
    // j: packed word column of the tile (0..WJ-1); rows rbase + kRowStep*i.
    // SwiGLU: the gate box holds words 0..WJ/2-1 and the up box the rest; each
    // warp stays on one box so its loads cover 128 contiguous bytes.
    int j, rbase, wbase, wstride;
    if (kGLU) {
      constexpr int WH = WJ / 2;
      const int half = gt / (kGT / 2), u = gt % (kGT / 2);
      j = half * WH + (u % WH);
      rbase = u / WH;
      wbase = half * (S::kWStage / 8) + (u % WH);
      wstride = WH;
    } else {
      j = gt % WJ;
      rbase = gt / WJ;
      wbase = j;
      wstride = WJ;
    }
    static_assert((kRowStep & (kRowStep - 1)) == 0, "row step is a power of two");
    // Row r = rbase + kRowStep*i splits into a per-thread part and a constant
    // part: r & 7 = (rbase & 7) | (kRowStep*i & 7) and r >> 3 = (rbase >> 3) +
    // (kRowStep*i >> 3) (no carries, kRowStep a power of two and rbase <
    // kRowStep or kRowStep a multiple of 8), so every store address is a
    // per-thread base + an immediate + one xor of the swizzled chunk.
    const int st_base = (j >> 3) * 8192 + (rbase >> 3) * 1024 + (rbase & 7) * 128;
    const int cx = (j & 7) ^ (rbase & 7);
    const int ld_base = wbase + rbase * wstride;
    const int jm = kGLU ? (j / (WJ / 2)) : mat;   // matrix of this column
    const int jw = kGLU ? (j % (WJ / 2)) : j;      // 8-feature word within the tile's slice
    int it0 = 0;  // first k-step of the current tile in this CTA's stream
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x, it0 += KB) {
      int e, mt, nt;
      decode(tile, e, mt, nt);
      const ExpertEntry* ent = table + e;
      const int n0 = nt * BO;
      const int g = ent->group_size;
      // this thread's 8 features: scales row stride N, zeros row stride N/8
      const bool jvalid = n0 + 8 * jw < N;
      const __half* scol = ent->scales[jm] + n0 + 8 * jw;
      const int32_t* zcol = ent->zeros[jm] + n0 / 8 + jw;
      auto load_params = [&](int kb, uint4& sc, uint32_t& zw) {
        const size_t grow = size_t((kb * kBK) / g);
        sc = make_uint4(0, 0, 0, 0);
        zw = 0;
        if (jvalid) {
          sc = __ldg(reinterpret_cast<const uint4*>(scol + grow * N));
          zw = uint32_t(__ldg(zcol + grow * (N / 8)));
        }
      };
      // this group's k-steps of the tile: kb = kb0, kb0 + DGROUPS, ...; the
      // scale / zero row of the next one is requested before the current one
      // is converted, so its latency hides behind a whole k-step
      int kb = DGROUPS > 1 ? (dgrp - it0 % DGROUPS + DGROUPS) % DGROUPS : 0;
      uint4 sc;
      uint32_t zw;
      if (kb < KB) load_params(kb, sc, zw);
      for (; kb < KB; kb += DGROUPS) {
        const int it = it0 + kb;
        uint4 sc_next = sc;
        uint32_t zw_next = zw;
        if (kb + DGROUPS < KB) load_params(kb + DGROUPS, sc_next, zw_next);
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        const int q = it % DSTAGES;
        const int prev = it - DSTAGES;  // last k-step that used buffer q
        if (!wait_any(&wfull[s], ph, s_abort, err) ||
            (prev >= 0 &&
             !wait_any(&empty[prev % STAGES], (prev / STAGES) & 1, s_abort, err))) {
          ok = false;
          break;
        }
        const uint32_t* w = sW + s * (S::kWStage / 4);
        DeqParams P;
        deq_params(zw, sc, P);
        uint8_t* bbuf = sB + q * S::kBBuf + st_base;
        const uint32_t* wrow = w + ld_base;
        // The packed words of a batch are all read before the first store: the
        // compiler cannot move a shared-memory load above a store it may alias,
        // and a load -> convert -> store chain per word would serialise on the
        // load latency.
        constexpr int kBatch = kWords < 8 ? kWords : 8;
#pragma unroll
        for (int i0 = 0; i0 < kWords; i0 += kBatch) {
          uint32_t wv[kBatch];
#pragma unroll
          for (int i = 0; i < kBatch; ++i) wv[i] = wrow[kRowStep * (i0 + i) * wstride];
#pragma unroll
          for (int i = 0; i < kBatch; ++i) {
            const int rk = kRowStep * (i0 + i);  // constant part of the row
            const uint4 o = deq_word(wv[i], P);
            *reinterpret_cast<uint4*>(bbuf + (rk >> 3) * 1024 + (rk & 7) * 128 +
                                      ((cx ^ (rk & 7)) << 4)) = o;
          }
        }
        // every packed word of the stage has been read and used: release it
        // to the weight producer before the operand buffer is published
        __syncwarp();
        if (lane == 0) mbar_arrive(&wempty[s]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dfull[q]);
        sc = sc_next;
        zw = zw_next;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int grp = warp >> 2;
    const int quarter = warp & 3;
    int lt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x, ++lt) {
      int e, mt, nt;
      decode(tile, e, mt, nt);
      const int acc = S::NACC == 2 ? (lt & 1) : 0;
      const uint32_t aph = S::NACC == 2 ? (lt >> 1) & 1 : lt & 1;
      // a group leaves together: the barrier reduces "any wait failed"
      const bool waited = wait_any(&tfull[acc], aph, s_abort, err);
      if (named_bar_any(1 + grp, !waited)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int rows_valid = min(ROWS, s_len[e] - mt * ROWS);
      const int row0 = s_start[e] + mt * ROWS;
      const int n0 = nt * BO;
      const uint32_t tacc = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * S::ACC);
      // TMEM lane = token row (M = 64: lanes 0-15 of each quarter), column =
      // weight column.  MT = 2: group g drains sub-tile g (all chunks); MT = 1:
      // the groups take alternate chunks.
      constexpr int RQ = S::RQ;
      const int msub = MT == 2 ? grp : 0;
      const int trow = msub * 128 + quarter * RQ + lane;  // token row within the tile
      const bool row_ok = lane < RQ && trow < rows_valid;
      __half* crow = C + size_t(row0 + (row_ok ? trow : 0)) * N;
      const uint32_t tbase = tacc + uint32_t(msub * WN);
      if (quarter * RQ < S::TOKROWS && msub * 128 + quarter * RQ < rows_valid) {
        // chunk c: accumulator columns 16c.. (SwiGLU: gate 16c.., up WN/2 + 16c..).
        // The loads of the next chunk are in flight while this one is converted
        // and stored.
        const int c0 = MT == 2 ? 0 : grp;
        constexpr int cstep = MT == 2 ? 1 : 2;
        const int cend = min(BO / 16, (N - n0 + 15) / 16);
        uint32_t v[16], u[16];
        if (c0 < cend) {
          tmem_ld_32x32b_x16(tbase + c0 * 16, v);
          if (kGLU) tmem_ld_32x32b_x16(tbase + WN / 2 + c0 * 16, u);
          tmem_ld_wait(v, u);
        }
        for (int c = c0; c < cend; c += cstep) {
          float f[16];
          if (kGLU) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              f[i] = silu_f32(__uint_as_float(v[i])) * __uint_as_float(u[i]);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              f[i] = __uint_as_float(v[i]);
              if (MODE == LR_FFN_MODE_SILU) f[i] = silu_f32(f[i]);
            }
          }
          const bool more = c + cstep < cend;
          if (more) {
            tmem_ld_32x32b_x16(tbase + (c + cstep) * 16, v);
            if (kGLU) tmem_ld_32x32b_x16(tbase + WN / 2 + (c + cstep) * 16, u);
          }
          if (row_ok) {
            uint4* dst = reinterpret_cast<uint4*>(crow + n0 + c * 16);
            dst[0] = pack8_feature_order(f);
            dst[1] = pack8_feature_order(f + 8);
          }
          if (more) tmem_ld_wait(v, u);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::NACC * S::ACC);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <class S, int MODE>
static int launch_gemm(const void* A, int K, int R, const ExpertEntry* table, int E, int mat,
                       int N, const int32_t* seg_start, const int32_t* seg_len, int max_rows,
                       __half* C, int32_t* err, cudaStream_t stream) {
  auto kern = w4a16_grouped_gemm_kernel<S, MODE>;
  static unsigned long long configured = 0;
  if (const int rc = set_dyn_smem_once(kern, S::kTotal, configured)) return rc;
  CUtensorMap ta;
  if (const int rc = encode_rows_cached(&ta, A, K, R, uint32_t(S::ROWS),
                                        CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  int sms = 0;
  if (const int rc = current_sm_count(&sms)) return rc;
  constexpr int BO = (MODE == LR_FFN_MODE_SWIGLU) ? S::WN / 2 : S::WN;
  const long n_tiles = (N + BO - 1) / BO;
  const long upper = long(E) * ((max_rows + S::ROWS - 1) / S::ROWS) * n_tiles;
  const int grid = int(upper < sms ? (upper < 1 ? 1 : upper) : sms);
  // token rows of an expert (max_rows x K fp16) against its weights (K x N / 2
  // bytes, twice for SwiGLU): keep the larger one's tiles shared by concurrent CTAs
  const long wcols = long(N) * (MODE == LR_FFN_MODE_SWIGLU ? 2 : 1);
  const int n_fastest = long(max_rows) * 4 > wcols ? 1 : 0;
  kern<<<grid, kGemmThreads, S::kTotal, stream>>>(ta, table, E, mat, K, N, seg_start, seg_len,
                                                  max_rows, R, C, err, n_fastest);
  LR_LAUNCH_CHECK();
  return LR_OK;
}

// Tile shape from the longest expert segment: 32 / 64 / 128 token rows with 256
// weight columns, or 256 token rows (two stacked M sub-tiles) with 128 weight
// columns (double-buffered accumulator) or, for long K, 256.
template <int MODE>
static int dispatch_shape(const void* A, int K, int R, const ExpertEntry* t, int E, int mat, int N,
                          const int32_t* ss, const int32_t* sl, int mr, __half* C, int32_t* err,
                          cudaStream_t st) {
  if (mr <= 32) return launch_gemm<ShapeR32, MODE>(A, K, R, t, E, mat, N, ss, sl, mr, C, err, st);
  if (mr <= 64) return launch_gemm<ShapeR64, MODE>(A, K, R, t, E, mat, N, ss, sl, mr, C, err, st);
  if (mr <= 128)
    return launch_gemm<ShapeR128, MODE>(A, K, R, t, E, mat, N, ss, sl, mr, C, err, st);
  if (K >= kWideTileMinK)
    return launch_gemm<ShapeR256W, MODE>(A, K, R, t, E, mat, N, ss, sl, mr, C, err, st);
  return launch_gemm<ShapeR256, MODE>(A, K, R, t, E, mat, N, ss, sl, mr, C, err, st);
}

}  // namespace lr

using namespace lr;

extern "C" size_t lr_weight_table_bytes(int num_experts) {
  return sizeof(ExpertEntry) * size_t(num_experts < 0 ? 0 : num_experts);
}

extern "C" int lr_encode_weight_table(const lr_expert_weights* experts, int E, int d_model,
                                      int d_ff, int group_size, int gated, void* host_table,
                                      size_t table_bytes) {
  if (!experts || E < 1 || E > kMaxGemmExperts || !host_table) return LR_ERR_INVALID_ARGUMENT;
  if (table_bytes < lr_weight_table_bytes(E)) return LR_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(host_table) & 127u) != 0) return LR_ERR_INVALID_ARGUMENT;
  if (group_size < 1) return LR_ERR_INVALID_ARGUMENT;
  ExpertEntry* tab = static_cast<ExpertEntry*>(host_table);
  memset(tab, 0, sizeof(ExpertEntry) * size_t(E));
  for (int e = 0; e < E; ++e) {
    ExpertEntry& ent = tab[e];
    ent.group_size = group_size;
    for (int m = 0; m < 3; ++m) {
      if (m == 0 && !gated) continue;
      const int K = (m < 2) ? d_model : d_ff;
      const int N = (m < 2) ? d_ff : d_model;
      const int32_t* qw = experts[e].qweight[m];
      if (!qw) continue;
      // the packed format's own limits (reference pack_weights.py:44-45)
      if (K < 1 || K % group_size != 0 || N < 8 || N % 8 != 0) return LR_ERR_UNSUPPORTED;
      if (!experts[e].scales[m] || !experts[e].zeros[m]) return LR_ERR_INVALID_ARGUMENT;
      if ((reinterpret_cast<uintptr_t>(qw) | reinterpret_cast<uintptr_t>(experts[e].scales[m]) |
           reinterpret_cast<uintptr_t>(experts[e].zeros[m])) & 15u)
        return LR_ERR_INVALID_ARGUMENT;
      // TMA strides are multiples of 16 bytes: N / 8 words per packed row
      if (N % 32 == 0) {
        CUtensorMap* maps[3] = {&ent.qw32[m], &ent.qw16[m], &ent.qw8[m]};
        const uint32_t words[3] = {32, 16, 8};
        for (int b = 0; b < 3; ++b) {
          const int rc = encode_2d(maps[b], CU_TENSOR_MAP_DATA_TYPE_INT32, qw, uint64_t(N / 8),
                                   uint64_t(K), uint64_t(N / 8) * 4, words[b], kBK,
                                   CU_TENSOR_MAP_SWIZZLE_NONE);
          if (rc) return rc;
        }
        ent.tma |= 1 << m;
      }
      ent.qw[m] = qw;
      ent.scales[m] = static_cast<const __half*>(experts[e].scales[m]);
      ent.zeros[m] = experts[e].zeros[m];
      ent.K[m] = K;
      ent.N[m] = N;
      ent.present |= 1 << m;
    }
  }
  return LR_OK;
}

extern "C" size_t lr_grouped_gemm_workspace_bytes(int num_experts) {
  (void)num_experts;
  return 0;
}

extern "C" size_t lr_grouped_w4a16_workspace_bytes(int num_experts, int R, int K, int N,
                                                   int group_size, int max_rows_per_expert) {
  if (num_experts < 1 || R < 1 || K < 1 || group_size < 1 || K % group_size != 0) return 0;
  if (!i8_eligible(K, N, group_size, max_rows_per_expert)) return 0;
  return i8_workspace_bytes(R, K);
}

extern "C" int lr_grouped_w4a16_gemm(const void* device_table, int E, int mode, int mat,
                                     const void* A, int R, int K, int N, int group_size,
                                     const int32_t* seg_start, const int32_t* seg_len,
                                     int max_rows_per_expert, void* C, void* workspace,
                                     size_t workspace_bytes, int32_t* err, lr_stream_t stream) {
  if (!device_table || E < 1 || E > kMaxGemmExperts) return LR_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(device_table) & 127u) != 0) return LR_ERR_INVALID_ARGUMENT;
  if (mode < LR_FFN_MODE_PLAIN || mode > LR_FFN_MODE_SWIGLU) return LR_ERR_INVALID_ARGUMENT;
  if (mode != LR_FFN_MODE_SWIGLU && (mat < 0 || mat > 2)) return LR_ERR_INVALID_ARGUMENT;
  if (K < 1 || group_size < 1 || K % group_size != 0) return LR_ERR_INVALID_ARGUMENT;
  if (N < 8 || N % 8 != 0) return LR_ERR_UNSUPPORTED;
  if (R < 0 || max_rows_per_expert < 0) return LR_ERR_INVALID_ARGUMENT;
  if (R == 0 || max_rows_per_expert == 0) return LR_OK;
  if (!A || !C || (reinterpret_cast<uintptr_t>(A) & 1u) || (reinterpret_cast<uintptr_t>(C) & 15u))
    return LR_ERR_INVALID_ARGUMENT;
  if ((seg_start == nullptr) != (seg_len == nullptr)) return LR_ERR_INVALID_ARGUMENT;
  if (!seg_start && E != 1) return LR_ERR_INVALID_ARGUMENT;
  const ExpertEntry* tab = static_cast<const ExpertEntry*>(device_table);
  __half* Cp = static_cast<__half*>(C);
  const int mr = max_rows_per_expert;
  const int g = group_size;
  // Kernel by shape: the tensor maps exist for N % 32 == 0; the token operand
  // goes through TMA when its rows are 16-byte aligned (K % 8 == 0).
  const bool tma = N % 32 == 0 && K % 8 == 0 && (reinterpret_cast<uintptr_t>(A) & 15u) == 0;
  const bool pow2_group = g >= 16 && (g & (g - 1)) == 0;
  int path = (tma && K % kBK == 0 && g % kBK == 0) ? 0 : (tma && pow2_group) ? 1 : 2;
  // short segments with a token-term workspace: 8-bit operands
  if (path == 0 && i8_eligible(K, N, g, mr) && workspace &&
      (reinterpret_cast<uintptr_t>(workspace) & 127u) == 0 &&
      workspace_bytes >= i8_workspace_bytes(R, K))
    path = 3;
#define LR_GEMM_MODE(M_)                                                                       \
  if (path == 3) return launch_i8<M_>(A, K, R, tab, E, mat, N, g, seg_start, seg_len, mr, Cp,   \
                                      workspace, err, stream);                                \
  if (path == 0) return dispatch_shape<M_>(A, K, R, tab, E, mat, N, seg_start, seg_len, mr, Cp, \
                                           err, stream);                                      \
  if (path == 1) return launch_skinny<M_>(A, K, R, tab, E, mat, N, seg_start, seg_len, mr, Cp,  \
                                          err, stream);                                       \
  return launch_generic<M_>(A, K, R, tab, E, mat, N, g, seg_start, seg_len, mr, Cp, err, stream)
  switch (mode) {
    case LR_FFN_MODE_PLAIN:
      LR_GEMM_MODE(LR_FFN_MODE_PLAIN);
    case LR_FFN_MODE_SILU:
      LR_GEMM_MODE(LR_FFN_MODE_SILU);
    default:
      LR_GEMM_MODE(LR_FFN_MODE_SWIGLU);
  }
#undef LR_GEMM_MODE
}

extern "C" int lr_quantized_matmul(const void* device_table, const void* A, int M, int K, int N,
                                   int group_size, void* C, void* workspace,
                                   size_t workspace_bytes, int32_t* err, lr_stream_t stream) {
  return lr_grouped_w4a16_gemm(device_table, 1, LR_FFN_MODE_PLAIN, 2, A, M, K, N, group_size,
                               nullptr, nullptr, M, C, workspace, workspace_bytes, err, stream);
}
