// lr_w4a16_gemm.cu -- grouped W4A16 expert GEMM on tcgen05 (sm_100a).
//
// Swap-AB formulation: for expert e and a tile of BM = 128 weight columns
// (output features) x BN tokens,
//     D[feature, token] = sum_k W[k, feature] * A[token, k]
// with W (dequantized INT4) as the UMMA "A" operand (M = 128, MN-major) and the
// token rows as the UMMA "B" operand (N = BN, K-major).  The accumulator lives
// in tensor memory (128 lanes = features, BN fp32 columns = tokens), double
// buffered so the epilogue of one tile overlaps the main loop of the next.
//
// Warp roles (576 threads, one CTA per SM, persistent over tiles):
//   warps 0-7   epilogue (two groups of four, alternate 16-token chunks):
//               tcgen05.ld -> activation -> fp16 -> staged in smem -> coalesced
//               16-byte stores (rows clipped to the expert segment)
//   warps 8-15  dequant: packed int32 words (TMA-staged) -> 8 fp16 each,
//               fp16(scale * (q - zero)) computed exactly, written into the
//               128-byte-swizzled MN-major operand buffer
//   warp 16     producer: TMA tile loads of tokens and packed weights (the
//               dequant warps read the per-group scales / zeros themselves)
//   warp 17     TMEM allocation + single-thread tcgen05.mma issue
//
// Every mbarrier wait is bounded in time; a wait that runs out raises a
// shared abort flag and LR_DEVERR_PIPE_TIMEOUT so all roles drain and exit.
#include <cudaTypedefs.h>
#include <cstring>

#include "lr_common.cuh"

namespace lr {

// ---------------------------------------------------------------------------
// per-expert weight table (device resident, written once per weight set)
// ---------------------------------------------------------------------------
struct alignas(128) ExpertEntry {
  CUtensorMap qw16[3];  // packed weights, box {16 words, 64 rows}
  CUtensorMap qw8[3];   // packed weights, box {8 words, 64 rows}
  const __half* scales[3];
  const int32_t* zeros[3];
  int32_t K[3];
  int32_t N[3];
  int32_t group_size;
  int32_t present;  // bit m set when matrix m is encoded
};
static_assert(sizeof(ExpertEntry) % 128 == 0, "table entry alignment");

constexpr int kEpiWarps = 8;
constexpr int kDeqWarps = 8;
constexpr int kProdWarp = kEpiWarps + kDeqWarps;
constexpr int kMmaWarp = kProdWarp + 1;
constexpr int kGemmThreads = (kMmaWarp + 1) * 32;
constexpr int kBK = 64;
constexpr int kMaxGemmExperts = 256;
constexpr int kABytes = 128 * kBK * 2;      // dequantized operand, one buffer
constexpr int kWBytes = kBK * 16 * 4;       // packed weights per stage (128 features)
constexpr int kCBytes = 6144;               // epilogue staging: [16][128] fp16, or [16][64] fp32 + [16][64] fp16
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s
constexpr uint64_t kDrainLimitNs = 100000000ull;  // 100 ms

template <int BN, int STAGES, int DSTAGES>
struct GemmLayout {
  static constexpr int kDStages = DSTAGES;
  static constexpr int kBStage = BN * 128;
  static constexpr int offB = 0;
  static constexpr int offA = offB + STAGES * kBStage;
  static constexpr int offW = offA + kDStages * kABytes;
  static constexpr int offC = offW + STAGES * kWBytes;
  static constexpr int offBar = offC + 2 * kCBytes;
  static constexpr int kNumBars = 2 * STAGES + 2 * kDStages + 4 + 1;
  static constexpr int offMisc = offBar + kNumBars * 8;
  static constexpr int kMiscInts = 8;
  static constexpr int offTab = offMisc + kMiscInts * 4;
  static constexpr int kTabBytes = (kMaxGemmExperts * 4 + 1) * 4;
  static constexpr int kTotal = offTab + kTabBytes + 1024;  // + base alignment slack
  static_assert(offA % 1024 == 0, "operand alignment");
};

// Pipeline depths per token tile: v = TMA stages (tokens + packed weights),
// d = dequantized-operand buffers.  Small tiles do little tensor work per k-step,
// so the dequant -> MMA -> release chain must be deeper to hide its latency.
template <int BN>
struct GemmStages;
template <>
struct GemmStages<16> { static constexpr int v = 16, d = 4; };
template <>
struct GemmStages<32> { static constexpr int v = 16, d = 4; };
template <>
struct GemmStages<64> { static constexpr int v = 10, d = 4; };
template <>
struct GemmStages<128> { static constexpr int v = 8, d = 2; };
template <>
struct GemmStages<256> { static constexpr int v = 4, d = 2; };

// ---------------------------------------------------------------------------
// int4 -> fp16 dequantization of one packed word (8 features)
// ---------------------------------------------------------------------------
LR_DEVICE uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// (w >> 4p) & 0x000F000F | 0x64006400: half2(1024 + nibble p, 1024 + nibble p+4).
LR_DEVICE uint32_t nib_pair(uint32_t w, int p) {
  uint32_t d;
  const uint32_t x = w >> (4 * p);
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(x), "r"(0x000F000Fu), "r"(0x64006400u));
  return d;
}

LR_DEVICE uint32_t h2_sub(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
LR_DEVICE uint32_t h2_mul(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

struct DeqParams {
  uint32_t z[4];  // half2(1024 + z_p, 1024 + z_{p+4})
  uint32_t s[4];  // half2(s_p, s_{p+4})
};

LR_DEVICE void deq_params(uint32_t zword, uint4 sc, DeqParams& P) {
#pragma unroll
  for (int p = 0; p < 4; ++p) P.z[p] = nib_pair(zword, p);
  P.s[0] = prmt(sc.x, sc.z, 0x5410);
  P.s[1] = prmt(sc.x, sc.z, 0x7632);
  P.s[2] = prmt(sc.y, sc.w, 0x5410);
  P.s[3] = prmt(sc.y, sc.w, 0x7632);
}

// fp16(scale * (q - z)): (1024+q) - (1024+z) is exact in fp16, and the product
// of an fp16 scale with an integer in [-15, 15] is rounded once.  The eight
// halves come out in the order f0 f4 f1 f5 f2 f6 f3 f7; the operand keeps that
// order (a permutation of the tile's M rows) and the epilogue maps each
// accumulator lane back to its feature with lane_feature().
LR_DEVICE uint4 deq_word(uint32_t w, const DeqParams& P) {
  uint4 o;
  o.x = h2_mul(h2_sub(nib_pair(w, 0), P.z[0]), P.s[0]);
  o.y = h2_mul(h2_sub(nib_pair(w, 1), P.z[1]), P.s[1]);
  o.z = h2_mul(h2_sub(nib_pair(w, 2), P.z[2]), P.s[2]);
  o.w = h2_mul(h2_sub(nib_pair(w, 3), P.z[3]), P.s[3]);
  return o;
}

// Feature (within its 8-feature group) held by accumulator lane `lane`.
LR_DEVICE int lane_feature(int lane) { return (lane & ~7) | ((lane & 7) >> 1) | ((lane & 1) << 2); }

// Named barrier over the 128 threads of one epilogue group.
LR_DEVICE void named_bar(int id) { asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory"); }

// Named barrier that also returns whether any of the 128 threads passed `pred`.
LR_DEVICE bool named_bar_any(int id, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.cta.red.or.pred q, %2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(pred)), "r"(id)
      : "memory");
  return r != 0;
}

LR_DEVICE bool wait_any(uint64_t* bar, uint32_t parity, volatile int* abort, int32_t* err) {
  return mbar_wait_bounded(bar, parity, abort, err, kWaitLimitNs);
}

// drain wait: ignores the abort flag, shorter limit, reports nothing
LR_DEVICE void wait_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > kDrainLimitNs) return;
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int BN, int STAGES, int DSTAGES, int MODE>
__global__ void __launch_bounds__(kGemmThreads, 1)
    w4a16_grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                              const ExpertEntry* __restrict__ table, int E, int mat, int K, int N,
                              const int32_t* __restrict__ seg_start,
                              const int32_t* __restrict__ seg_len, int max_rows, int R,
                              __half* __restrict__ C, int32_t* err) {
  using L = GemmLayout<BN, STAGES, DSTAGES>;
  constexpr int kDStages = DSTAGES;
  constexpr int BO = (MODE == LR_FFN_MODE_SWIGLU) ? 64 : 128;  // output features per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sB = smem + L::offB;
  uint8_t* sA = smem + L::offA;
  uint32_t* sW = reinterpret_cast<uint32_t*>(smem + L::offW);
  uint8_t* sC = smem + L::offC;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::offBar);
  uint64_t* empty = full + STAGES;
  uint64_t* dfull = empty + STAGES;
  uint64_t* dempty = dfull + kDStages;
  uint64_t* tfull = dempty + kDStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* fin = tempty + 2;
  int* misc = reinterpret_cast<int*>(smem + L::offMisc);
  volatile int* s_abort = misc;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(misc + 1);
  int* s_tbase = reinterpret_cast<int*>(smem + L::offTab);  // E+1
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
    }
    for (int i = 0; i < kDStages; ++i) {
      mbar_init(&dfull[i], kDeqWarps / kDStages);
      mbar_init(&dempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kEpiWarps * 32);
    }
    mbar_init(fin, 1);
    *s_abort = 0;
    fence_mbarrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(s_tmem, 2 * BN);
    tmem_relinquish();
  }
  if (warp == kProdWarp) {
    if (lane == 0) tma_prefetch_desc(&tmap_a);
    int carry = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      int st = 0, len = 0;
      if (e < E) {
        if (seg_start) {
          st = __ldg(seg_start + e);
          len = __ldg(seg_len + e);
        } else {
          st = 0;
          len = R;
        }
        if (len < 0) len = 0;
        if (len > max_rows) {
          report(err, LR_DEVERR_BAD_SEGMENT);
          len = max_rows;
        }
        if (st < 0 || st + len > R) {
          report(err, LR_DEVERR_BAD_SEGMENT);
          st = 0;
          len = 0;
        }
      }
      const int mt = (len + BN - 1) / BN;
      const int tiles = mt * n_tiles;
      int incl = tiles;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int x = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += x;
      }
      if (e < E) {
        s_tbase[e] = carry + incl - tiles;
        s_start[e] = st;
        s_len[e] = len;
        s_mt[e] = mt;
      }
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) s_tbase[E] = carry;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int total = s_tbase[E];

  auto decode = [&](int tile, int& e, int& mt, int& nt) {
    int lo = 0, hi = E;  // last e with s_tbase[e] <= tile
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_tbase[mid] <= tile) lo = mid;
      else hi = mid;
    }
    e = lo;
    const int local = tile - s_tbase[e];
    nt = local / s_mt[e];
    mt = local - nt * s_mt[e];
  };

  if (warp == kProdWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
        int e, mt, nt;
        decode(tile, e, mt, nt);
        const ExpertEntry* ent = table + e;
        const int row0 = s_start[e] + mt * BN;
        const int n0 = nt * BO;
        const CUtensorMap* wmap0 = (MODE == LR_FFN_MODE_SWIGLU) ? &ent->qw8[0] : &ent->qw16[mat];
        const CUtensorMap* wmap1 = &ent->qw8[1];
        // descriptors were written to global memory by a copy before the launch
        tensormap_acquire(wmap0);
        if (MODE == LR_FFN_MODE_SWIGLU) tensormap_acquire(wmap1);
        // Only the token box and the packed weight box(es) travel by TMA: each
        // copy costs issue time on this single thread, so the small per-group
        // scale / zero rows are read by the dequant warps themselves.
        const uint32_t tx = uint32_t(BN * 128 + kWBytes);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!wait_any(&empty[s], ph ^ 1, s_abort, err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], tx);
          tma_load_2d(sB + s * L::kBStage, &tmap_a, &full[s], kb * kBK, row0);
          uint32_t* w = sW + s * (kWBytes / 4);
          tma_load_2d(w, wmap0, &full[s], n0 / 8, kb * kBK);
          if (MODE == LR_FFN_MODE_SWIGLU) tma_load_2d(w + 512, wmap1, &full[s], n0 / 8, kb * kBK);
        }
      }
      if (ok) {
        // Producer tail: wait until the MMA has released every stage.  The
        // releases are tcgen05.commit arrivals that complete asynchronously;
        // leaving before they land would let them hit the barriers of the next
        // CTA placed on this SM.
        for (int i = 0; i < STAGES; ++i, ++it) {
          if (!wait_any(&empty[it % STAGES], ((it / STAGES) & 1) ^ 1, s_abort, err)) break;
        }
      } else {
        // let in-flight copies land before the CTA exits
        const int first = it - STAGES < 0 ? 0 : it - STAGES;
        for (int i = first; i < it; ++i) wait_drain(&full[i % STAGES], (i / STAGES) & 1);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(128, BN, 1, 0);
      int it = 0, lt = 0;
      bool ok = true;
      // Readiness of k-step `it` observed ahead of time: the barriers of the
      // next k-step are tested (non-blocking) before this k-step's MMAs are
      // issued, so the test latency overlaps the MMA issue instead of adding
      // to it; a blocking wait is needed only when the test came back false.
      bool pre_full = false, pre_dfull = false;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x, ++lt) {
        const int acc = lt & 1;
        const uint32_t aph = (lt >> 1) & 1;
        if (!wait_any(&tempty[acc], aph ^ 1, s_abort, err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          const int q = it % kDStages;
          const uint32_t qph = (it / kDStages) & 1;
          if ((!pre_full && !wait_any(&full[s], ph, s_abort, err)) ||
              (!pre_dfull && !wait_any(&dfull[q], qph, s_abort, err))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int it2 = it + 1;  // next k-step of this CTA's stream (maybe the next tile's)
          const bool more = kb + 1 < KB || tile + int(gridDim.x) < total;
          const bool nf = more && mbar_test_wait(&full[it2 % STAGES], (it2 / STAGES) & 1);
          const bool nd = more && mbar_test_wait(&dfull[it2 % kDStages], (it2 / kDStages) & 1);
          const uint32_t aaddr = smem_u32(sA + q * kABytes);
          const uint32_t baddr = smem_u32(sB + s * L::kBStage);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t adesc = umma_smem_desc(aaddr + kk * 2048, 8192, 1024, 2);
            const uint64_t bdesc = umma_smem_desc(baddr + kk * 32, 16, 1024, 2);
            umma_f16_ss(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[s]);
          umma_commit(&dempty[q]);
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
    // The dequant warps form kDStages groups of kWg warps; group g converts
    // the k-steps it with it % kDStages == g into operand buffer g, so that
    // kDStages k-steps (each a dependent load -> convert -> store -> fence
    // chain) are in flight at once.
    constexpr int kWg = kDeqWarps / kDStages;     // warps per group
    constexpr int kGT = 32 * kWg;                 // threads per group
    constexpr int kWords = 1024 / kGT;            // packed words per thread per k-step
    constexpr int kRowStep = kGT / 16;            // rows between a thread's words
    const int dtid = threadIdx.x - kEpiWarps * 32;
    const int dgrp = dtid / kGT;
    const int gt = dtid % kGT;
    // j: packed word column of the 128-feature tile (0..15); rows rbase + kRowStep*i.
    // SwiGLU keeps each warp on one box (gate or up), so a warp's loads cover
    // contiguous bytes instead of two same-bank pieces.
    int j, rbase, wbase, wstride;
    if (MODE == LR_FFN_MODE_SWIGLU) {
      const int half = gt / (kGT / 2), u = gt % (kGT / 2);
      j = half * 8 + (u & 7);
      rbase = u >> 3;
      wbase = half * 512 + (u & 7);
      wstride = 8;
    } else {
      j = gt & 15;
      rbase = gt >> 4;
      wbase = j;
      wstride = 16;
    }
    const int chunk = j & 7;
    const int jm = (MODE == LR_FFN_MODE_SWIGLU) ? (j >> 3) : mat;  // matrix of this column
    const int jw = (MODE == LR_FFN_MODE_SWIGLU) ? (j & 7) : j;      // word within the tile
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
      int e, mt, nt;
      decode(tile, e, mt, nt);
      const ExpertEntry* ent = table + e;
      const int n0 = nt * BO;
      const int g = ent->group_size;
      // this thread's 8 features: scales row stride N, zeros row stride N/8
      const bool jvalid = n0 + 8 * jw < N;
      const __half* scol = ent->scales[jm] + n0 + 8 * jw;
      const int32_t* zcol = ent->zeros[jm] + n0 / 8 + jw;
      for (int kb = 0; kb < KB; ++kb, ++it) {
        if (it % kDStages != dgrp) continue;
        const size_t grow = size_t((kb * kBK) / g);
        uint4 sc = make_uint4(0, 0, 0, 0);
        uint32_t zw = 0;
        if (jvalid) {  // issued before the waits so their latency overlaps them
          sc = __ldg(reinterpret_cast<const uint4*>(scol + grow * N));
          zw = uint32_t(__ldg(zcol + grow * (N / 8)));
        }
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        const int q = dgrp;
        const uint32_t qph = (it / kDStages) & 1;
        if (!wait_any(&full[s], ph, s_abort, err) || !wait_any(&dempty[q], qph ^ 1, s_abort, err)) {
          ok = false;
          break;
        }
        const uint32_t* w = sW + s * (kWBytes / 4);
        DeqParams P;
        deq_params(zw, sc, P);
        uint8_t* abuf = sA + q * kABytes + (j >> 3) * 8192;
#pragma unroll
        for (int i = 0; i < kWords; ++i) {
          const int r = rbase + kRowStep * i;
          const uint4 o = deq_word(w[wbase + r * wstride], P);
          *reinterpret_cast<uint4*>(abuf + (r >> 3) * 1024 + (r & 7) * 128 +
                                    ((chunk ^ (r & 7)) << 4)) = o;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dfull[q]);
      }
    }
    // Dequant tail: the group's operand buffer is released by an asynchronous
    // tcgen05.commit arrival; wait for the last one before the CTA can exit.
    for (int i = 0; ok && i < kDStages; ++i, ++it) {
      if (it % kDStages != dgrp) continue;
      if (!wait_any(&dempty[dgrp], ((it / kDStages) & 1) ^ 1, s_abort, err)) break;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Two groups of four warps; warp w reads TMEM lanes 32*(w%4).. and group
    // w/4 takes every other 16-column chunk, with its own named barrier and
    // staging buffer.
    const int grp = warp >> 2;
    const int bar_id = 1 + grp;
    const int etid = (warp & 3) * 32 + lane;    // 0..127 == TMEM lane
    const int fe = lane_feature(etid);          // feature of this lane within the tile
    const int fe64 = lane_feature(etid & 63);   // SwiGLU: gate/up feature of this lane
    uint8_t* sCg = sC + grp * kCBytes;
    int lt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x, ++lt) {
      int e, mt, nt;
      decode(tile, e, mt, nt);
      const int acc = lt & 1;
      const uint32_t aph = (lt >> 1) & 1;
      // a group leaves together: the barrier reduces "any wait failed"
      const bool waited = wait_any(&tfull[acc], aph, s_abort, err);
      if (named_bar_any(bar_id, !waited)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int row_base = s_start[e] + mt * BN;
      const int rows_valid = min(BN, s_len[e] - mt * BN);
      const int n0 = nt * BO;
      const uint32_t tbase =
          tmem_base + (uint32_t((warp & 3) * 32) << 16) + uint32_t(acc * BN);
      for (int c = grp; c < BN / 16; c += 2) {
        if (c * 16 >= rows_valid) break;
        uint32_t v[16];
        tmem_ld_32x32b_x16_sync(tbase + c * 16, v);
        const int nrow = min(16, rows_valid - c * 16);
        if (MODE != LR_FFN_MODE_SWIGLU) {
          __half* stage = reinterpret_cast<__half*>(sCg);  // [16][128]
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            float f = __uint_as_float(v[jj]);
            if (MODE == LR_FFN_MODE_SILU) f = silu_f32(f);
            stage[jj * 128 + fe] = __float2half_rn(f);
          }
          named_bar(bar_id);
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int idx = etid + i * 128;
            const int row = idx >> 4, ch = idx & 15;
            if (row < nrow && n0 + ch * 8 < N) {
              *reinterpret_cast<uint4*>(C + size_t(row_base + c * 16 + row) * N + n0 + ch * 8) =
                  *reinterpret_cast<const uint4*>(sCg + row * 256 + ch * 16);
            }
          }
          named_bar(bar_id);
        } else {
          float* sU = reinterpret_cast<float*>(sCg);                // [16][64] fp32
          __half* stage = reinterpret_cast<__half*>(sCg + 4096);    // [16][64] fp16
          if (etid >= 64) {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) sU[jj * 64 + fe64] = __uint_as_float(v[jj]);
          }
          named_bar(bar_id);
          if (etid < 64) {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const float gv = __uint_as_float(v[jj]);
              const float uv = sU[jj * 64 + fe64];
              stage[jj * 64 + fe64] = __float2half_rn(silu_f32(gv) * uv);
            }
          }
          named_bar(bar_id);
          {
            const int row = etid >> 3, ch = etid & 7;
            if (row < nrow) {
              *reinterpret_cast<uint4*>(C + size_t(row_base + c * 16 + row) * N + n0 + ch * 8) =
                  *reinterpret_cast<const uint4*>(sCg + 4096 + row * 128 + ch * 16);
            }
          }
          named_bar(bar_id);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

static int encode_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t dim0,
                     uint64_t dim1, uint64_t stride1_bytes, uint32_t box0, uint32_t box1,
                     CUtensorMapSwizzle sw) {
  auto fn = get_encode_fn();
  if (!fn) return LR_ERR_NO_DEVICE;
  const cuuint64_t dims[2] = {dim0, dim1};
  const cuuint64_t strides[1] = {stride1_bytes};
  const cuuint32_t box[2] = {box0, box1};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LR_OK : LR_ERR_INVALID_ARGUMENT;
}

template <int BN, int MODE>
static int launch_gemm(const CUtensorMap& tmap_a, const ExpertEntry* table, int E, int mat, int K,
                       int N, const int32_t* seg_start, const int32_t* seg_len, int max_rows, int R,
                       __half* C, int32_t* err, cudaStream_t stream) {
  constexpr int STAGES = GemmStages<BN>::v;
  constexpr int DSTAGES = GemmStages<BN>::d;
  using L = GemmLayout<BN, STAGES, DSTAGES>;
  static_assert(L::kTotal <= 227 * 1024, "shared memory budget");
  auto kern = w4a16_grouped_gemm_kernel<BN, STAGES, DSTAGES, MODE>;
  static int configured = 0;
  if (!configured) {
    LR_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal));
    configured = 1;
  }
  int dev = 0, sms = 0;
  LR_CUDA_TRY(cudaGetDevice(&dev));
  LR_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  constexpr int BO = (MODE == LR_FFN_MODE_SWIGLU) ? 64 : 128;
  const long n_tiles = (N + BO - 1) / BO;
  const long upper = long(E) * ((max_rows + BN - 1) / BN) * n_tiles;
  const int grid = int(upper < sms ? (upper < 1 ? 1 : upper) : sms);
  kern<<<grid, kGemmThreads, L::kTotal, stream>>>(tmap_a, table, E, mat, K, N, seg_start, seg_len,
                                                  max_rows, R, C, err);
  LR_LAUNCH_CHECK();
  return LR_OK;
}

template <int MODE>
static int dispatch_bn(int BN, const CUtensorMap& ta, const ExpertEntry* t, int E, int mat, int K,
                       int N, const int32_t* ss, const int32_t* sl, int mr, int R, __half* C,
                       int32_t* err, cudaStream_t st) {
  switch (BN) {
    case 16: return launch_gemm<16, MODE>(ta, t, E, mat, K, N, ss, sl, mr, R, C, err, st);
    case 32: return launch_gemm<32, MODE>(ta, t, E, mat, K, N, ss, sl, mr, R, C, err, st);
    case 64: return launch_gemm<64, MODE>(ta, t, E, mat, K, N, ss, sl, mr, R, C, err, st);
    case 128: return launch_gemm<128, MODE>(ta, t, E, mat, K, N, ss, sl, mr, R, C, err, st);
    default: return launch_gemm<256, MODE>(ta, t, E, mat, K, N, ss, sl, mr, R, C, err, st);
  }
}

static int pick_bn(int max_rows) {
  if (max_rows <= 16) return 16;
  if (max_rows <= 32) return 32;
  if (max_rows <= 64) return 64;
  if (max_rows <= 128) return 128;
  return 256;
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
  if (group_size < kBK || group_size % kBK != 0) return LR_ERR_UNSUPPORTED;
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
      if (K % kBK != 0 || K % group_size != 0 || N % 32 != 0) return LR_ERR_UNSUPPORTED;
      if (!experts[e].scales[m] || !experts[e].zeros[m]) return LR_ERR_INVALID_ARGUMENT;
      if ((reinterpret_cast<uintptr_t>(qw) | reinterpret_cast<uintptr_t>(experts[e].scales[m]) |
           reinterpret_cast<uintptr_t>(experts[e].zeros[m])) & 15u)
        return LR_ERR_INVALID_ARGUMENT;
      int rc = encode_2d(&ent.qw16[m], CU_TENSOR_MAP_DATA_TYPE_INT32, qw, uint64_t(N / 8),
                         uint64_t(K), uint64_t(N / 8) * 4, 16, kBK, CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc) return rc;
      rc = encode_2d(&ent.qw8[m], CU_TENSOR_MAP_DATA_TYPE_INT32, qw, uint64_t(N / 8), uint64_t(K),
                     uint64_t(N / 8) * 4, 8, kBK, CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc) return rc;
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

extern "C" int lr_grouped_w4a16_gemm(const void* device_table, int E, int mode, int mat,
                                     const void* A, int R, int K, int N, const int32_t* seg_start,
                                     const int32_t* seg_len, int max_rows_per_expert, void* C,
                                     void* workspace, size_t workspace_bytes, int32_t* err,
                                     lr_stream_t stream) {
  (void)workspace;
  (void)workspace_bytes;
  if (!device_table || E < 1 || E > kMaxGemmExperts) return LR_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(device_table) & 127u) != 0) return LR_ERR_INVALID_ARGUMENT;
  if (mode < LR_FFN_MODE_PLAIN || mode > LR_FFN_MODE_SWIGLU) return LR_ERR_INVALID_ARGUMENT;
  if (mode != LR_FFN_MODE_SWIGLU && (mat < 0 || mat > 2)) return LR_ERR_INVALID_ARGUMENT;
  if (K < kBK || K % kBK != 0) return LR_ERR_UNSUPPORTED;
  if (N < 32 || N % (mode == LR_FFN_MODE_SWIGLU ? 64 : 32) != 0) return LR_ERR_UNSUPPORTED;
  if (R < 0 || max_rows_per_expert < 0) return LR_ERR_INVALID_ARGUMENT;
  if (R == 0 || max_rows_per_expert == 0) return LR_OK;
  if (!A || !C || ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(C)) & 15u))
    return LR_ERR_INVALID_ARGUMENT;
  if ((seg_start == nullptr) != (seg_len == nullptr)) return LR_ERR_INVALID_ARGUMENT;
  if (!seg_start && E != 1) return LR_ERR_INVALID_ARGUMENT;
  const int BN = pick_bn(max_rows_per_expert);
  CUtensorMap ta;
  int rc = encode_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, A, uint64_t(K), uint64_t(R),
                     uint64_t(K) * 2, kBK, uint32_t(BN), CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const ExpertEntry* tab = static_cast<const ExpertEntry*>(device_table);
  __half* Cp = static_cast<__half*>(C);
  switch (mode) {
    case LR_FFN_MODE_PLAIN:
      return dispatch_bn<LR_FFN_MODE_PLAIN>(BN, ta, tab, E, mat, K, N, seg_start, seg_len,
                                            max_rows_per_expert, R, Cp, err, stream);
    case LR_FFN_MODE_SILU:
      return dispatch_bn<LR_FFN_MODE_SILU>(BN, ta, tab, E, mat, K, N, seg_start, seg_len,
                                           max_rows_per_expert, R, Cp, err, stream);
    default:
      return dispatch_bn<LR_FFN_MODE_SWIGLU>(BN, ta, tab, E, mat, K, N, seg_start, seg_len,
                                             max_rows_per_expert, R, Cp, err, stream);
  }
}

extern "C" int lr_quantized_matmul(const void* device_table, const void* A, int M, int K, int N,
                                   void* C, void* workspace, size_t workspace_bytes, int32_t* err,
                                   lr_stream_t stream) {
  return lr_grouped_w4a16_gemm(device_table, 1, LR_FFN_MODE_PLAIN, 2, A, M, K, N, nullptr,
                               nullptr, M, C, workspace, workspace_bytes, err, stream);
}
