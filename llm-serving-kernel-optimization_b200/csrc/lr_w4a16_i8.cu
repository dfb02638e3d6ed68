// lr_w4a16_i8.cu -- grouped W4A16 expert GEMM for short expert segments
// (decode), on 8-bit tcgen05 operands (sm_100a).
//
// At decode an expert sees at most a few dozen token rows, so the GEMM is a
// stream of packed INT4 weights.  With fp16 operands every weight is written to
// and read from shared memory as two bytes and the tensor core spends a whole
// instruction on each 16-deep slice.  This kernel feeds the tensor core 8-bit
// operands instead (half the operand bytes, twice the depth per instruction):
//
//   weights  the INT4 codes q in [0, 15] themselves, as unsigned bytes (exact).
//            Unpacking a packed word is two masks and a shift: the low nibbles
//            of a word become bytes 0..3, the high nibbles bytes 4..7.
//   tokens   each row, per block of 128 k, as two signed 8-bit terms:
//            x ~= sigma * (a1 + a2 / 256) with sigma = max|x| / 127 of the block,
//            a1 = round(x / sigma), a2 = round(256 * (x - sigma * a1) / sigma).
//            The reconstruction error is at most sigma / 512 per element (16-bit
//            fixed point relative to the block maximum), or sigma / 256 where the
//            residual sits at +-sigma / 2 and a2 saturates at +-127.
//
// The weights are the UMMA A operand (M = 128 weight rows, MN-major), the two
// token terms of up to 32 rows the B operand (N = 64, K-major).  The group
// scale and zero cannot ride inside an 8-bit code, so every 128-deep block gets
// its own int32 accumulator, and the epilogue warps fold it into fp32 sums:
//
//   y[t, n] += (sigma_t / 256) * s[g, n] * (256 * A1 + A2 - z[g, n] * X_t)
//
// with A1 = sum_k a1 * q, A2 = sum_k a2 * q (exact int32) and
// X_t = sum_k (256 * a1 + a2) over the block.  This is sum_k x~ * s * (q - z):
// the weights enter as s * (q - z) exactly, where the reference rounds them to
// fp16 first (lightning_router/quantization/pack_weights.py:89-105); the
// difference is below fp16 resolution of each weight.
//
// Warp roles (640 threads, one CTA per SM, persistent over tiles of one expert
// x 256 weight rows):
//   warps 0-7   epilogue: per block, tcgen05.ld of the int32 accumulators, the
//               fold above into fp32 registers (thread = weight row); after the
//               last block the activation and fp16 stores
//   warps 8-15  unpack: packed words (TMA-staged) -> bytes, written into the
//               128-byte-swizzled MN-major operand buffer of their block
//   warp 16     token producer: TMA loads of the two term boxes
//   warp 17     weight producer: TMA loads of the packed weight boxes
//   warp 18     TMEM allocation + single-thread tcgen05.mma (kind::i8) issue
//   warp 19     parameter producer: the block's (sigma, X) of every token row and
//               scale and zero of every weight row, read with plain loads two
//               blocks ahead and stored into the block's parameter slot (small
//               TMA copies would queue in front of the weight boxes)
//
// Every mbarrier wait is bounded in time; a wait that runs out raises a shared
// abort flag and LR_DEVERR_PIPE_TIMEOUT so all roles drain and exit.
#include "lr_w4a16.cuh"

namespace lr {

namespace i8 {

constexpr int kQK = 128;       // k per block (activation block, pipeline step, accumulator)
constexpr int kRows = 32;      // token rows per tile
constexpr int kBN = 2 * kRows; // B operand rows: term 1 of every row, then term 2
constexpr int kWM = 256;       // weight rows per tile: two M = 128 halves
constexpr int kEpiWarps = 8;
constexpr int kUnpWarps = 8;
constexpr int kTokWarp = kEpiWarps + kUnpWarps;
constexpr int kWgtWarp = kTokWarp + 1;
constexpr int kMmaWarp = kWgtWarp + 1;
constexpr int kParWarp = kMmaWarp + 1;
constexpr int kThreads = (kParWarp + 1) * 32;

constexpr int STAGES = 3;   // token stages (released by the MMA)
constexpr int WSTAGES = 5;  // packed-weight stages (released by the unpack warps)
constexpr int DSTAGES = 3;  // unpacked operand buffers (released by the MMA)
constexpr int NACC = 4;     // int32 accumulators of 2 x 64 TMEM columns
constexpr int NP = 16;      // parameter slots (released by the epilogue)
constexpr int kAccCols = 2 * kBN;
constexpr int kTmemCols = NACC * kAccCols;

constexpr int kDBuf = kWM * kQK;        // unpacked operand: 2 halves x 128 rows x 128 k
constexpr int kTStage = kBN * kQK;      // token terms: 64 rows x 128 bytes
constexpr int kWStage = kQK * kWM / 2;  // packed words of a block
// parameter slot: sigma[32] (fp32), X[32] (int32), the scales of the tile's
// 256 weight rows (fp16) and their packed zeros (32 words)
constexpr int kPSig = 0, kPX = kRows * 4, kPScale = 2 * kRows * 4, kPZero = kPScale + kWM * 2;
constexpr int kPSlot = kPZero + kWM / 2;

constexpr int offD = 0;
constexpr int offT = offD + DSTAGES * kDBuf;
constexpr int offW = offT + STAGES * kTStage;
constexpr int offP = offW + WSTAGES * kWStage;
constexpr int offBar = offP + NP * kPSlot;
constexpr int kNumBars = 2 * STAGES + 2 * WSTAGES + 2 * DSTAGES + 2 * NACC + 2 * NP + 1;
constexpr int offMisc = offBar + kNumBars * 8;
constexpr int offTab = offMisc + 8 * 4;
constexpr int kTabBytes = (kMaxGemmExperts * 4 + 1) * 4;
constexpr int kTotal = offTab + kTabBytes + 1024;  // + base alignment slack
static_assert(offD % 1024 == 0 && offT % 1024 == 0 && kDBuf % 1024 == 0 &&
                  kTStage % 1024 == 0,
              "128-byte swizzled operands start on 1024-byte boundaries");
static_assert(offW % 128 == 0 && kWStage % 128 == 0, "TMA destinations are 128-byte aligned");
static_assert(offP % 128 == 0 && kPSlot % 128 == 0 && kPScale % 16 == 0 && kPZero % 16 == 0,
              "parameter slots hold 16-byte vectors");
static_assert(kTotal <= 227 * 1024, "shared memory budget");
static_assert(kTmemCols <= 512, "TMEM columns");

// Instruction descriptor, kind::i8: D int32, A unsigned 8-bit MN-major
// (weights), B signed 8-bit K-major (token terms), M = 128, N = kBN.
constexpr uint32_t kIdesc = (2u << 4)               // D format s32
                            | (0u << 7)             // A unsigned 8-bit
                            | (1u << 10)            // B signed 8-bit
                            | (1u << 15)            // A MN-major
                            | (0u << 16)            // B K-major
                            | (uint32_t(kBN >> 3) << 17) | (uint32_t(128 >> 4) << 24);

LR_DEVICE void umma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 bit, 4 consecutive columns per thread (asynchronous: consume
// after tmem_wait4 on the same arrays).
LR_DEVICE void tmem_ld_x4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr)
               : "memory");
}
LR_DEVICE void tmem_ld_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
LR_DEVICE void tmem_wait8(uint32_t (&a)[8], uint32_t (&b)[8], uint32_t (&c)[8],
                          uint32_t (&d)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]),
                 "+r"(a[6]), "+r"(a[7]), "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]),
                 "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]), "+r"(c[0]), "+r"(c[1]),
                 "+r"(c[2]), "+r"(c[3]), "+r"(c[4]), "+r"(c[5]), "+r"(c[6]), "+r"(c[7]),
                 "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3]), "+r"(d[4]), "+r"(d[5]),
                 "+r"(d[6]), "+r"(d[7])
               :
               : "memory");
}
LR_DEVICE void tmem_wait4(uint32_t (&a)[4], uint32_t (&b)[4], uint32_t (&c)[4],
                          uint32_t (&d)[4]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(b[0]), "+r"(b[1]),
                 "+r"(b[2]), "+r"(b[3]), "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3]),
                 "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
               :
               : "memory");
}

// Bytes 0..15 of an unpacked 16-feature chunk hold features
// 0 2 4 6 1 3 5 7 8 10 12 14 9 11 13 15 (low nibbles of the first word, its
// high nibbles, then the second word): the feature at operand row position b.
LR_DEVICE int chunk_feature(int b) { return (b & 8) | ((b & 3) << 1) | ((b >> 2) & 1); }

}  // namespace i8

// ---------------------------------------------------------------------------
// token rows -> two 8-bit terms per 128-k block
// ---------------------------------------------------------------------------
// One warp per (row r, block j); lane l holds elements 4l .. 4l+3 of the block.
// Aq: term 1 of row r at row r, term 2 at row R + r (2R rows of K bytes);
// sig[j * R + r] = sigma / 256, xs[j * R + r] = sum (256 * a1 + a2).
__global__ void __launch_bounds__(256)
    quantize_rows_i8x2_kernel(const __half* __restrict__ A, int R, int K,
                              int8_t* __restrict__ Aq, float* __restrict__ sig,
                              int32_t* __restrict__ xs) {
  pdl_wait();
  pdl_trigger();
  const int KB = K / i8::kQK;
  const int lane = threadIdx.x & 31;
  const long total = long(R) * KB;
  const long nwarps = long(gridDim.x) * (blockDim.x >> 5);
  for (long u = long(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); u < total;
       u += nwarps) {
    const int r = int(u / KB), j = int(u - long(r) * KB);
    const size_t off = size_t(r) * K + size_t(j) * i8::kQK + 4 * lane;
    const uint2 raw = __ldg(reinterpret_cast<const uint2*>(A + off));
    const float2 x01 = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
    const float2 x23 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
    const float x[4] = {x01.x, x01.y, x23.x, x23.y};
    float m = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float sigma = m / 127.0f;
    const float inv = m > 0.0f ? 127.0f / m : 0.0f;
    uint32_t w1 = 0, w2 = 0;
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float q1 = fminf(fmaxf(rintf(x[i] * inv), -127.0f), 127.0f);
      const float rr = fmaf(-q1, sigma, x[i]);
      const float q2 = fminf(fmaxf(rintf(rr * inv * 256.0f), -127.0f), 127.0f);
      const int a1 = int(q1), a2 = int(q2);
      w1 |= (uint32_t(a1) & 0xFFu) << (8 * i);
      w2 |= (uint32_t(a2) & 0xFFu) << (8 * i);
      sum += 256 * a1 + a2;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    *reinterpret_cast<uint32_t*>(Aq + off) = w1;
    *reinterpret_cast<uint32_t*>(Aq + size_t(R) * K + off) = w2;
    if (lane == 0) {
      sig[size_t(j) * R + r] = sigma * (1.0f / 256.0f);
      xs[size_t(j) * R + r] = sum;
    }
  }
}

// ---------------------------------------------------------------------------
// the GEMM
// ---------------------------------------------------------------------------
template <int MODE>
__global__ void __launch_bounds__(i8::kThreads, 1)
    w4a16_i8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_q,
                         const ExpertEntry* __restrict__ table, int E, int mat, int K, int N,
                         int group_size, const int32_t* __restrict__ seg_start,
                         const int32_t* __restrict__ seg_len, int max_rows, int R,
                         const float* __restrict__ sig, const int32_t* __restrict__ xsum,
                         __half* __restrict__ C, int32_t* err) {
  using namespace i8;
  constexpr bool kGLU = MODE == LR_FFN_MODE_SWIGLU;
  constexpr int BO = kGLU ? kWM / 2 : kWM;  // output features per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sD = smem + offD;
  uint8_t* sT = smem + offT;
  uint32_t* sW = reinterpret_cast<uint32_t*>(smem + offW);
  uint8_t* sP = smem + offP;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + offBar);  // token stage loaded
  uint64_t* empty = full + STAGES;       // token stage released by the MMA
  uint64_t* wfull = empty + STAGES;      // packed stage loaded
  uint64_t* wempty = wfull + WSTAGES;    // packed stage read by the unpack warps
  uint64_t* dfull = wempty + WSTAGES;    // unpacked operand written
  uint64_t* dempty = dfull + DSTAGES;    // unpacked operand released by the MMA
  uint64_t* tfull = dempty + DSTAGES;    // accumulator complete
  uint64_t* tempty = tfull + NACC;       // accumulator read by the epilogue
  uint64_t* pfull = tempty + NACC;       // parameter slot written
  uint64_t* pempty = pfull + NP;         // parameter slot read by the epilogue
  uint64_t* fin = pempty + NP;
  int* misc = reinterpret_cast<int*>(smem + offMisc);
  volatile int* s_abort = misc;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(misc + 1);
  int* s_tbase = reinterpret_cast<int*>(smem + offTab);  // E+1
  int* s_start = s_tbase + E + 1;
  int* s_len = s_start + E;
  int* s_mt = s_len + E;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (N + BO - 1) / BO;
  const int KB = K / kQK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < WSTAGES; ++i) {
      mbar_init(&wfull[i], 1);
      mbar_init(&wempty[i], kUnpWarps);
    }
    for (int i = 0; i < DSTAGES; ++i) {
      mbar_init(&dfull[i], kUnpWarps);
      mbar_init(&dempty[i], 1);
    }
    for (int i = 0; i < NACC; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kEpiWarps);
    }
    for (int i = 0; i < NP; ++i) {
      mbar_init(&pfull[i], 1);
      mbar_init(&pempty[i], kEpiWarps);
    }
    mbar_init(fin, 1);
    *s_abort = 0;
    fence_mbarrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(s_tmem, kTmemCols);
    tmem_relinquish();
  }
  if (warp == kTokWarp && lane == 0) tma_prefetch_desc(&tmap_q);
  // everything above touches only shared and tensor memory; the segments, token
  // terms and parameters below are the predecessors' outputs
  pdl_wait();
  pdl_trigger();
  if (warp == kTokWarp) {
    build_tile_table(seg_start, seg_len, E, R, max_rows, kRows, n_tiles, s_tbase, s_start, s_len,
                     s_mt, err);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int total = s_tbase[E];

  auto decode = [&](int tile, int& e, int& mt, int& nt) {
    decode_tile(s_tbase, s_mt, E, tile, e, mt, nt);
  };

  if (warp == kTokWarp) {
    // ------------------------------------------------------------ token producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
        int e, mt, nt;
        decode(tile, e, mt, nt);
        const int row0 = s_start[e] + mt * kRows;
        for (int j = 0; j < KB; ++j, ++it) {
          const int s = it % STAGES;
          if (!wait_any(&empty[s], ((it / STAGES) & 1) ^ 1, s_abort, err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], uint32_t(kTStage));
          uint8_t* dst = sT + s * kTStage;
          tma_load_2d(dst, &tmap_q, &full[s], j * kQK, row0);                    // term 1
          tma_load_2d(dst + kTStage / 2, &tmap_q, &full[s], j * kQK, R + row0);  // term 2
        }
      }
      if (ok) {
        // wait until the MMA has released every stage: its tcgen05.commit
        // arrivals land asynchronously and must not reach the barriers of the
        // next CTA placed on this SM
        for (int i = 0; i < STAGES; ++i, ++it) {
          if (!wait_any(&empty[it % STAGES], ((it / STAGES) & 1) ^ 1, s_abort, err)) break;
        }
      } else {
        const int first = it - STAGES < 0 ? 0 : it - STAGES;
        for (int i = first; i < it; ++i) wait_drain(&full[i % STAGES], (i / STAGES) & 1);
      }
    }
  } else if (warp == kParWarp) {
    // ------------------------------------------------------------ parameter producer
    // This CTA's blocks form one stream: block `it` is k-block it % KB of tile
    // blockIdx.x + (it / KB) * gridDim.x.
    const int my_tiles = total > int(blockIdx.x) ? (total - int(blockIdx.x) + int(gridDim.x) - 1) /
                                                         int(gridDim.x)
                                                   : 0;
    const int nblk = my_tiles * KB;
    struct Params {
      float sg;
      int xv;
      uint4 sc;     // 8 scales of this lane's weight rows
      uint32_t zw;  // their packed zeros
    };
    // the tile of the block being loaded: token row, scale and zero columns
    int ctile = -1, crow = 0;
    bool cvalid = false;
    const __half* cscale = nullptr;
    const int32_t* czero = nullptr;
    // parameters of block `it` into registers (stored two blocks later)
    auto pload = [&](int it, Params& r) {
      const int tile = int(blockIdx.x) + (it / KB) * int(gridDim.x);
      const int j = it % KB;
      if (tile != ctile) {
        int e, mt, nt;
        decode(tile, e, mt, nt);
        ctile = tile;
        crow = s_start[e] + mt * kRows + lane;
        // lane l: weight rows 8l .. 8l+7 of the tile (SwiGLU: lanes 0-15 gate,
        // 16-31 up, for the same 128 features)
        const int m = kGLU ? (lane >> 4) : mat;
        const int col = nt * BO + 8 * (kGLU ? (lane & 15) : lane);
        cvalid = col < N;
        const ExpertEntry* ent = table + e;
        cscale = ent->scales[m] + col;
        czero = ent->zeros[m] + col / 8;
      }
      r.sg = 0.0f;
      r.xv = 0;
      if (crow < R) {
        r.sg = __ldg(sig + size_t(j) * R + crow);
        r.xv = __ldg(xsum + size_t(j) * R + crow);
      }
      const size_t grp = size_t(j) * kQK / group_size;
      r.sc = make_uint4(0, 0, 0, 0);
      r.zw = 0;
      if (cvalid) {
        r.sc = __ldg(reinterpret_cast<const uint4*>(cscale + grp * N));
        r.zw = uint32_t(__ldg(czero + grp * (N / 8)));
      }
    };
    auto store = [&](int it, const Params& r) -> bool {
      const int p = it % NP;
      bool w = true;
      if (lane == 0) w = wait_any(&pempty[p], ((it / NP) & 1) ^ 1, s_abort, err);
      if (!__shfl_sync(0xffffffffu, int(w), 0)) return false;
      uint8_t* ps = sP + p * kPSlot;
      reinterpret_cast<float*>(ps + kPSig)[lane] = r.sg;
      reinterpret_cast<int*>(ps + kPX)[lane] = r.xv;
      reinterpret_cast<uint4*>(ps + kPScale)[lane] = r.sc;
      reinterpret_cast<uint32_t*>(ps + kPZero)[lane] = r.zw;
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfull[p]);
      return true;
    };
    Params ra, rb;
    if (nblk > 0) pload(0, ra);
    if (nblk > 1) pload(1, rb);
    for (int it = 0; it < nblk; it += 2) {
      if (!store(it, ra)) break;
      if (it + 2 < nblk) pload(it + 2, ra);
      if (it + 1 < nblk) {
        if (!store(it + 1, rb)) break;
        if (it + 3 < nblk) pload(it + 3, rb);
      }
    }
  } else if (warp == kWgtWarp) {
    // ------------------------------------------------------------ weight producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
        int e, mt, nt;
        decode(tile, e, mt, nt);
        const ExpertEntry* ent = table + e;
        const int n0 = nt * BO;
        const int x0 = n0 / 8;  // first packed word column
        const CUtensorMap* m0 = kGLU ? &ent->qw16[0] : &ent->qw32[mat];
        const CUtensorMap* m1 = &ent->qw16[1];
        // descriptors were written to global memory by a copy before the launch
        tensormap_acquire(m0);
        if (kGLU) tensormap_acquire(m1);
        for (int j = 0; j < KB; ++j, ++it) {
          const int s = it % WSTAGES;
          if (!wait_any(&wempty[s], ((it / WSTAGES) & 1) ^ 1, s_abort, err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&wfull[s], uint32_t(kWStage));
          uint32_t* w = sW + s * (kWStage / 4);
          // PLAIN / SILU: rows of 32 words; SwiGLU: 128 rows x 16 gate words,
          // then 128 rows x 16 up words (each box is 64 rows)
          if (kGLU) {
            tma_load_2d(w, m0, &wfull[s], x0, j * kQK);
            tma_load_2d(w + 64 * 16, m0, &wfull[s], x0, j * kQK + 64);
            tma_load_2d(w + 128 * 16, m1, &wfull[s], x0, j * kQK);
            tma_load_2d(w + 192 * 16, m1, &wfull[s], x0, j * kQK + 64);
          } else {
            tma_load_2d(w, m0, &wfull[s], x0, j * kQK);
            tma_load_2d(w + 64 * 32, m0, &wfull[s], x0, j * kQK + 64);
          }
        }
      }
      // the last copies (which the unpack warps may not wait for after an
      // abort) land before the CTA exits
      (void)ok;
      const int first = it - WSTAGES < 0 ? 0 : it - WSTAGES;
      for (int i = first; i < it; ++i) wait_drain(&wfull[i % WSTAGES], (i / WSTAGES) & 1);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      // Readiness of the next block observed ahead of time: its barriers are
      // tested (non-blocking) before this block's MMAs are issued, so a
      // blocking wait -- whose wake-up latency would leave the tensor pipe
      // idle -- is needed only when a test came back false.
      bool pre_t = false, pre_f = false, pre_d = false;
      for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
        for (int j = 0; j < KB; ++j, ++it) {
          const int b = it % NACC, s = it % STAGES, q = it % DSTAGES;
          if ((!pre_t && !wait_any(&tempty[b], ((it / NACC) & 1) ^ 1, s_abort, err)) ||
              (!pre_f && !wait_any(&full[s], (it / STAGES) & 1, s_abort, err)) ||
              (!pre_d && !wait_any(&dfull[q], (it / DSTAGES) & 1, s_abort, err))) {
            ok = false;
            break;
          }
          tc_fence_after();
          {
            const int n = it + 1;
            const bool more = j + 1 < KB || tile + int(gridDim.x) < total;
            pre_t = more && mbar_test_wait(&tempty[n % NACC], ((n / NACC) & 1) ^ 1);
            pre_f = more && mbar_test_wait(&full[n % STAGES], (n / STAGES) & 1);
            pre_d = more && mbar_test_wait(&dfull[n % DSTAGES], (n / DSTAGES) & 1);
          }
          const uint32_t aaddr = smem_u32(sD + q * kDBuf);
          const uint32_t baddr = smem_u32(sT + s * kTStage);
          const uint32_t d = tmem_base + uint32_t(b * kAccCols);
#pragma unroll
          for (int kk = 0; kk < kQK / 32; ++kk) {
            // token terms: K-major rows of 128 bytes, 32 bytes per instruction
            const uint64_t bdesc = umma_smem_desc(baddr + kk * 32, 16, 1024, 2);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              // weights: MN-major, one 128-byte atom of M per k row, 32 k rows
              // per instruction
              const uint64_t adesc =
                  umma_smem_desc(aaddr + h * (kDBuf / 2) + kk * 4096, kDBuf / 2, 1024, 2);
              umma_i8_ss(d + uint32_t(h * kBN), adesc, bdesc, kIdesc, kk != 0 ? 1u : 0u);
            }
          }
          umma_commit(&empty[s]);
          umma_commit(&dempty[q]);
          umma_commit(&tfull[b]);
        }
      }
      if (!ok) {
        umma_commit(fin);
        wait_drain(fin, 0);
      }
    }
  } else if (warp >= kEpiWarps) {
    // ------------------------------------------------------------ unpack
    const int ut = threadIdx.x - kEpiWarps * 32;  // 0..255
    // chunk c (16 features: two packed words) and first row of this thread.
    // PLAIN: a half-warp reads one 128-byte packed row; SwiGLU: a quarter-warp
    // reads 64 bytes of gate (or up) words, two rows per half-warp, so the
    // loads of a half-warp cover all 32 banks.  The stores of a quarter-warp
    // cover the eight 16-byte chunks of one operand row.
    int c, rsub, src;
    if (kGLU) {
      const int cc = ut & 7, rp = (ut >> 3) & 1, hh = (ut >> 4) & 1;
      c = cc + 8 * hh;
      rsub = rp + 2 * (ut >> 5);
      src = hh * (128 * 16) + rsub * 16 + 2 * cc;
    } else {
      c = ut & 15;
      rsub = ((ut >> 4) & 1) + 2 * (ut >> 5);
      src = rsub * 32 + 2 * c;
    }
    constexpr int kRowWords = kGLU ? 16 : 32;
    const int dst = (c >> 3) * (kDBuf / 2) + rsub * 128 + (((c & 7) ^ (rsub & 7)) << 4);
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
      for (int j = 0; j < KB; ++j, ++it) {
        const int s = it % WSTAGES, q = it % DSTAGES;
        // lane 0 polls the barriers for its warp (every lane polling would
        // add a shared-memory operation per lane per block); __syncwarp then
        // orders the other lanes' reads after its acquire
        bool w = true;
        if (lane == 0)
          w = wait_any(&wfull[s], (it / WSTAGES) & 1, s_abort, err) &&
              wait_any(&dempty[q], ((it / DSTAGES) & 1) ^ 1, s_abort, err);
        if (!__shfl_sync(0xffffffffu, int(w), 0)) {
          ok = false;
          break;
        }
        __syncwarp();
        const uint32_t* wsrc = sW + s * (kWStage / 4) + src;
        uint2 wv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          wv[i] = *reinterpret_cast<const uint2*>(wsrc + 16 * i * kRowWords);
        uint8_t* d = sD + q * kDBuf + dst;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          uint4 o;
          o.x = wv[i].x & 0x0F0F0F0Fu;
          o.y = (wv[i].x >> 4) & 0x0F0F0F0Fu;
          o.z = wv[i].y & 0x0F0F0F0Fu;
          o.w = (wv[i].y >> 4) & 0x0F0F0F0Fu;
          // rows rsub + 16i keep the swizzle phase (rsub & 7) of the thread
          *reinterpret_cast<uint4*>(d + i * 16 * 128) = o;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&wempty[s]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dfull[q]);
      }
    }
    if (ok && lane == 0) {
      // the MMA's releases of the last buffers land before the CTA exits
      for (int u = it - DSTAGES < 0 ? 0 : it - DSTAGES; u < it; ++u)
        if (!wait_any(&dempty[u % DSTAGES], (u / DSTAGES) & 1, s_abort, err)) break;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3, gsel = warp >> 2;
    const int L = quarter * 32 + lane;  // TMEM lane = operand row within a half
    const int fpos = (L & ~15) | chunk_feature(L & 15);
    const uint32_t tlane = tmem_base + (uint32_t(quarter * 32) << 16);
    int it = 0;
    bool ok = true;
    bool pre_a = false, pre_p = false;
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
      int e, mt, nt;
      decode(tile, e, mt, nt);
      const int rows_valid = min(kRows, s_len[e] - mt * kRows);
      const int row0 = s_start[e] + mt * kRows;
      const int n0 = nt * BO;
      int f[2];
      f[0] = n0 + fpos;
      f[1] = kGLU ? f[0] : n0 + 128 + fpos;
      const bool fv0 = f[0] < N, fv1 = f[1] < N;
      float run[2][16];
#pragma unroll
      for (int i = 0; i < 16; ++i) run[0][i] = run[1][i] = 0.0f;
      for (int j = 0; j < KB; ++j, ++it) {
        const int b = it % NACC, p = it % NP;
        // lane 0 polls for its warp (see the unpack warps)
        bool w = true;
        if (lane == 0)
          w = (pre_a || wait_any(&tfull[b], (it / NACC) & 1, s_abort, err)) &&
              (pre_p || wait_any(&pfull[p], (it / NP) & 1, s_abort, err));
        if (!__shfl_sync(0xffffffffu, int(w), 0)) {
          ok = false;
          break;
        }
        __syncwarp();
        tc_fence_after();
        if (lane == 0) {
          // the next block's barriers, tested while this one is folded
          const int n = it + 1;
          const bool more = j + 1 < KB || tile + int(gridDim.x) < total;
          pre_a = more && mbar_test_wait(&tfull[n % NACC], (n / NACC) & 1);
          pre_p = more && mbar_test_wait(&pfull[n % NP], (n / NP) & 1);
        }
        const uint8_t* ps = sP + p * kPSlot;
        // scale and -zero of this thread's two weight rows (tile row L and 128 + L)
        const __half* pscale = reinterpret_cast<const __half*>(ps + kPScale);
        const uint32_t* pzero = reinterpret_cast<const uint32_t*>(ps + kPZero);
        const float sc0 = __half2float(pscale[fpos]);
        const float sc1 = __half2float(pscale[128 + fpos]);
        const int nz0 = -int((pzero[fpos >> 3] >> (4 * (fpos & 7))) & 15u);
        const int nz1 = -int((pzero[16 + (fpos >> 3)] >> (4 * (fpos & 7))) & 15u);
        const float* psig = reinterpret_cast<const float*>(ps + kPSig);
        const int* pxs = reinterpret_cast<const int*>(ps + kPX);
        const uint32_t tb = tlane + uint32_t(b * kAccCols);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int t0 = 8 * (2 * i + gsel);  // this thread's rows t0 .. t0+7
          if (t0 < rows_valid) {
            uint32_t a1[8], a2[8], u1[8], u2[8];
            tmem_ld_x8(tb + t0, a1);                 // half 0, term 1
            tmem_ld_x8(tb + kRows + t0, a2);         // half 0, term 2
            tmem_ld_x8(tb + kBN + t0, u1);           // half 1, term 1
            tmem_ld_x8(tb + kBN + kRows + t0, u2);   // half 1, term 2
            const float4 sga = *reinterpret_cast<const float4*>(psig + t0);
            const float4 sgb = *reinterpret_cast<const float4*>(psig + t0 + 4);
            const int4 xva = *reinterpret_cast<const int4*>(pxs + t0);
            const int4 xvb = *reinterpret_cast<const int4*>(pxs + t0 + 4);
            const float sgv[8] = {sga.x, sga.y, sga.z, sga.w, sgb.x, sgb.y, sgb.z, sgb.w};
            const int xvv[8] = {xva.x, xva.y, xva.z, xva.w, xvb.x, xvb.y, xvb.z, xvb.w};
            tmem_wait8(a1, a2, u1, u2);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const int v0 = int(a1[u]) * 256 + int(a2[u]) + nz0 * xvv[u];
              const int v1 = int(u1[u]) * 256 + int(u2[u]) + nz1 * xvv[u];
              run[0][8 * i + u] = fmaf(float(v0), sgv[u] * sc0, run[0][8 * i + u]);
              run[1][8 * i + u] = fmaf(float(v1), sgv[u] * sc1, run[1][8 * i + u]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&tempty[b]);
          mbar_arrive(&pempty[p]);
        }
      }
      if (!ok) break;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int t = 8 * (2 * i + gsel) + u;
          if (t < rows_valid) {
            __half* crow = C + size_t(row0 + t) * N;
            const float g0 = run[0][8 * i + u], g1 = run[1][8 * i + u];
            if (kGLU) {
              if (fv0) crow[f[0]] = __float2half_rn(silu_f32(g0) * g1);
            } else {
              const float o0 = MODE == LR_FFN_MODE_SILU ? silu_f32(g0) : g0;
              const float o1 = MODE == LR_FFN_MODE_SILU ? silu_f32(g1) : g1;
              if (fv0) crow[f[0]] = __float2half_rn(o0);
              if (fv1) crow[f[1]] = __float2half_rn(o1);
            }
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static size_t align128(size_t b) { return (b + 127) & ~size_t(127); }

size_t i8_workspace_bytes(int R, int K) {
  const size_t KB = size_t(K) / i8::kQK;
  return align128(size_t(2) * R * K) + 2 * align128(size_t(4) * R * KB);
}

bool i8_eligible(int K, int N, int group_size, int max_rows) {
  return max_rows >= 1 && max_rows <= i8::kRows && K % i8::kQK == 0 && group_size % i8::kQK == 0 &&
         N % 32 == 0;
}

// Tensor map of the token terms (2R rows of K bytes, box 128 x 32, 128-byte
// swizzle), reused while the same host thread passes the same workspace.
static int encode_terms_cached(CUtensorMap* out, const void* q, int K, int R) {
  struct Entry {
    const void* q;
    int K, R, dev;
    CUtensorMap map;
  };
  thread_local Entry cache[4];
  thread_local int used = 0, next = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return LR_ERR_NO_DEVICE;
  for (int i = 0; i < used; ++i) {
    const Entry& c = cache[i];
    if (c.q == q && c.K == K && c.R == R && c.dev == dev) {
      *out = c.map;
      return LR_OK;
    }
  }
  const int rc = encode_2d(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, uint64_t(K), uint64_t(2) * R,
                           uint64_t(K), i8::kQK, i8::kRows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  cache[next] = Entry{q, K, R, dev, *out};
  next = (next + 1) % 4;
  if (used < 4) ++used;
  return LR_OK;
}

template <int MODE>
int launch_i8(const void* A, int K, int R, const ExpertEntry* table, int E, int mat, int N,
              int group_size, const int32_t* seg_start, const int32_t* seg_len, int max_rows,
              __half* C, void* ws, int32_t* err, cudaStream_t stream) {
  const int KB = K / i8::kQK;
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  int8_t* q = reinterpret_cast<int8_t*>(wsb);
  float* sig = reinterpret_cast<float*>(wsb + align128(size_t(2) * R * K));
  int32_t* xs = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(sig) +
                                           align128(size_t(4) * R * KB));
  int sms = 0;
  if (const int rc = current_sm_count(&sms)) return rc;
  {
    const long warps = long(R) * KB;
    long blocks = (warps + 7) / 8;
    if (blocks > long(sms) * 16) blocks = long(sms) * 16;
    if (const int rc = launch_pdl(quantize_rows_i8x2_kernel, dim3(unsigned(blocks)), dim3(256), 0,
                                  stream, static_cast<const __half*>(A), R, K, q, sig, xs))
      return rc;
  }
  auto kern = w4a16_i8_gemm_kernel<MODE>;
  static unsigned long long configured = 0;
  if (const int rc = set_dyn_smem_once(kern, i8::kTotal, configured)) return rc;
  CUtensorMap tq;
  if (const int rc = encode_terms_cached(&tq, q, K, R)) return rc;
  constexpr int BO = (MODE == LR_FFN_MODE_SWIGLU) ? i8::kWM / 2 : i8::kWM;
  const long n_tiles = (N + BO - 1) / BO;
  const long upper = long(E) * ((max_rows + i8::kRows - 1) / i8::kRows) * n_tiles;
  const int grid = int(upper < sms ? (upper < 1 ? 1 : upper) : sms);
  if (const int rc = launch_pdl(kern, dim3(grid), dim3(i8::kThreads), size_t(i8::kTotal), stream,
                               tq, table, E, mat, K, N, group_size, seg_start, seg_len, max_rows,
                               R, static_cast<const float*>(sig), static_cast<const int32_t*>(xs),
                               C, err))
    return rc;
  return LR_OK;
}

template int launch_i8<LR_FFN_MODE_PLAIN>(const void*, int, int, const ExpertEntry*, int, int,
                                          int, int, const int32_t*, const int32_t*, int, __half*,
                                          void*, int32_t*, cudaStream_t);
template int launch_i8<LR_FFN_MODE_SILU>(const void*, int, int, const ExpertEntry*, int, int, int,
                                         int, const int32_t*, const int32_t*, int, __half*, void*,
                                         int32_t*, cudaStream_t);
template int launch_i8<LR_FFN_MODE_SWIGLU>(const void*, int, int, const ExpertEntry*, int, int,
                                           int, int, const int32_t*, const int32_t*, int, __half*,
                                           void*, int32_t*, cudaStream_t);

}  // namespace lr
