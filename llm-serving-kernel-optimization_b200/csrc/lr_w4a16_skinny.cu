// lr_w4a16_skinny.cu -- grouped W4A16 expert GEMM for short expert segments
// (decode-sized: at most 32 token rows per expert).
//
// At a few token rows per expert the GEMM is a weight stream: every packed INT4
// word is used by <= 32 tokens.  The tcgen05 path turns each weight into an fp16
// operand in shared memory (written by CUDA cores, read by the tensor core) and
// its per-instruction cost does not shrink with the 64-row UMMA it has to use,
// so it moves ~5 bytes of shared memory per weight.  Here the weights are the M
// operand of mma.sync.m16n8k16 and are dequantized straight into the A
// fragment registers: shared memory carries only the TMA-staged packed words
// (half a byte per weight, written once, read once) and the token box.
//
// Unit of work (one CTA): one expert, one tile of TR token rows, one slab of
// weight columns (NB boxes of 64 columns; SwiGLU: NB/2 gate boxes and the same
// features' NB/2 up boxes) over the whole K.  A CTA is NB*KSPLIT = 8 warps,
// two CTAs per SM.  Warp w dequantizes box w % NB on the 16-deep k slices
// w / NB, w / NB + KSPLIT, ... of every 64-deep stage.
//
// Stages (a STAGES ring) are TMA loads of the token box (TR rows x 64 k fp16,
// 128-byte swizzle) and the NB packed-weight boxes (64 k rows x 8 words).  There
// is no producer warp: thread 0 fills the ring at the start, and the last warp
// to finish a stage (a shared-memory counter with acquire-release semantics)
// refills its slot with the stage STAGES ahead.  A lane's per-group scale and
// zero words (16 + 4 bytes for its 8 features) are plain loads issued one group
// ahead of their use (one-row TMA boxes for them stalled the ring).
//
// Dequantization is the reference's single rounding fp16(scale * (q - zero))
// (lightning_router/quantization/pack_weights.py:119-130): two packed words (k
// and k+1) are interleaved by byte permutes so that one LOP3 yields
// half2(1024 + q_k, 1024 + q_k+1) (low nibbles) or half2(1024 + 16 q_k, ...)
// (high nibbles); q - z then comes exactly from one HSUB2 (or one HFMA2 by
// 1/16 for the high form) and one HMUL2 by the group scale rounds once.
//
// The KSPLIT warps of a box hold partial sums of interleaved k slices; they are
// added in warp order through shared memory, so a row's result depends only on
// K, the group size and its own inputs (not on the grid or the other rows).
//
// Every mbarrier wait is bounded in time; a wait that runs out raises a shared
// abort flag and LR_DEVERR_PIPE_TIMEOUT, the producer lets its copies land, and
// the CTA exits without writing outputs.
#include <type_traits>

#include "lr_w4a16.cuh"

namespace lr {

template <int NB_, int KSPLIT_, int TR_, int STAGES_>
struct SkinnyShape {
  static constexpr int NB = NB_, KSPLIT = KSPLIT_, TR = TR_, STAGES = STAGES_;
  static constexpr int kConsumers = NB * KSPLIT;
  static constexpr int kThreads = kConsumers * 32;
  static constexpr int NT = TR / 8;                 // token n tiles
  static constexpr int kAcc = 16 * NT;              // fp32 accumulators per lane
  static constexpr int kTokBytes = TR * 128;        // TR rows x 64 k fp16
  static constexpr int kBoxBytes = kBK * 8 * 4;     // 64 k rows x 8 words
  static constexpr int offW = kTokBytes;
  static constexpr int kStageBytes = (offW + NB * kBoxBytes + 1023) / 1024 * 1024;
  static constexpr int kRing = STAGES * kStageBytes;
  // reduction scratch (reuses the ring once the last stage is consumed)
  static constexpr int kRedSlots = (KSPLIT - 1) * NB > NB / 2 ? (KSPLIT - 1) * NB : NB / 2;
  static constexpr int kRedBytes = kRedSlots * 32 * kAcc * 4;
  static constexpr int offBar = kRing;
  static constexpr int kTotal = offBar + 2 * STAGES * 8 + STAGES * 4 + 16 + 1024;  // + slack
  static_assert(kConsumers == 8, "8 warps: two CTAs per SM, warps even over the SM's quarters");
  static_assert(offW % 128 == 0 && kBoxBytes % 128 == 0 && kStageBytes % 1024 == 0,
                "tiled TMA destinations are 128-byte aligned (the token box 1024)");
  static_assert(TR % 8 == 0 && TR >= 8 && TR <= 32, "token rows");
  static_assert(4 % KSPLIT == 0, "k slices per stage split evenly");
  static_assert(kRedBytes <= kRing, "reduction scratch fits in the ring");
  static_assert(2 * kTotal <= 227 * 1024, "two CTAs per SM");
};

LR_DEVICE void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                           uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
LR_DEVICE void ldmatrix_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}

LR_DEVICE void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

LR_DEVICE uint32_t lop3_ea(uint32_t x, uint32_t mask) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(x), "r"(mask), "r"(0x64006400u));
  return d;
}
LR_DEVICE uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
  __half2 r = __hfma2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b),
                      *reinterpret_cast<__half2*>(&c));
  return *reinterpret_cast<uint32_t*>(&r);
}

// Per-group dequantization constants of a lane's 8 features.
struct SkParams {
  uint32_t zlo[4];  // features 0,2,4,6: half2(1024 + z, 1024 + z)
  uint32_t zhi[4];  // features 1,3,5,7: half2(-(64 + z), -(64 + z))
  uint32_t s[8];    // half2(s_f, s_f)
};

LR_DEVICE void sk_params(uint32_t zw, uint4 sc, SkParams& P) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t z0 = (zw >> (8 * i)) & 0xFu, z1 = (zw >> (8 * i + 4)) & 0xFu;
    P.zlo[i] = 0x64006400u | z0 | (z0 << 16);
    const __half2 h = __float2half2_rn(-(64.0f + float(z1)));
    P.zhi[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  const uint32_t w[4] = {sc.x, sc.y, sc.z, sc.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    P.s[2 * i] = prmt(w[i], w[i], 0x1010);
    P.s[2 * i + 1] = prmt(w[i], w[i], 0x3232);
  }
}

// x = bytes {w_k.b0, w_k.b1, w_k1.b0, w_k1.b1} (or .b2/.b3): the nibbles of
// features f0..f0+3 at k (low half) and k+1 (high half).  out[j] =
// half2(W[k][f0+j], W[k+1][f0+j]).
LR_DEVICE void sk_deq4(uint32_t x, const SkParams& P, int f0, uint32_t (&out)[4]) {
  const uint32_t one16 = 0x2C002C00u;  // half2(1/16, 1/16)
  const uint32_t x8 = x >> 8;
  out[0] = h2_mul(h2_sub(lop3_ea(x, 0x000F000Fu), P.zlo[f0 / 2]), P.s[f0]);
  out[1] = h2_mul(h2_fma(lop3_ea(x, 0x00F000F0u), one16, P.zhi[f0 / 2]), P.s[f0 + 1]);
  out[2] = h2_mul(h2_sub(lop3_ea(x8, 0x000F000Fu), P.zlo[f0 / 2 + 1]), P.s[f0 + 2]);
  out[3] = h2_mul(h2_fma(lop3_ea(x8, 0x00F000F0u), one16, P.zhi[f0 / 2 + 1]), P.s[f0 + 3]);
}

LR_DEVICE bool bar_any(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.cta.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(pred)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

LR_DEVICE uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
LR_DEVICE uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// Shared-memory fetch-and-add with acquire-release semantics at CTA scope.
LR_DEVICE uint32_t atom_add_acq_rel(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;"
               : "=r"(old)
               : "r"(smem_u32(p)), "r"(v)
               : "memory");
  return old;
}

// Two CTAs per SM (8 warps each): 112 registers per thread.
template <class S, int MODE>
__global__ void __maxnreg__(112)
    w4a16_skinny_kernel(const __grid_constant__ CUtensorMap tmap_a,
                        const ExpertEntry* __restrict__ table, int E, int mat, int K, int N,
                        const int32_t* __restrict__ seg_start,
                        const int32_t* __restrict__ seg_len, int max_rows, int R, int n_slabs,
                        int m_tiles, __half* __restrict__ C, int32_t* err) {
  constexpr int NB = S::NB, KSPLIT = S::KSPLIT, TR = S::TR, NT = S::NT, STAGES = S::STAGES;
  constexpr bool kGLU = MODE == LR_FFN_MODE_SWIGLU;
  constexpr int BO = kGLU ? NB * 32 : NB * 64;  // output features of a unit
  static_assert(!kGLU || NB % 2 == 0, "SwiGLU pairs gate and up boxes");

  // unit -> (expert, token tile, feature slab); feature slabs vary fastest so
  // CTAs running together share the expert's token rows through L2
  const int slab = blockIdx.x % n_slabs;
  const int rest = blockIdx.x / n_slabs;
  const int mt = rest % m_tiles;
  const int e = rest / m_tiles;
  if (e >= E) return;
  int st = seg_start ? __ldg(seg_start + e) : 0;
  int len = seg_start ? __ldg(seg_len + e) : R;
  if (len < 0) len = 0;
  if (len > max_rows) {
    if (threadIdx.x == 0 && mt == 0 && slab == 0) report(err, LR_DEVERR_BAD_SEGMENT);
    len = max_rows;
  }
  if (st < 0 || st + len > R) {
    if (threadIdx.x == 0 && mt == 0 && slab == 0) report(err, LR_DEVERR_BAD_SEGMENT);
    return;
  }
  const int rows_valid = min(TR, len - mt * TR);
  if (rows_valid <= 0) return;  // the whole CTA leaves together
  const int row0 = st + mt * TR;
  const int f0 = slab * BO;  // first output feature (SwiGLU) / weight column (plain)

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::offBar);
  uint32_t* done = reinterpret_cast<uint32_t*>(full + STAGES);  // warps finished per slot
  volatile int* s_abort = reinterpret_cast<volatile int*>(done + STAGES);
  int* s_issued = const_cast<int*>(s_abort) + 1;                 // stages issued so far

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = (K + kBK - 1) / kBK;
  const ExpertEntry* ent = table + e;
  // group of a 16-deep slice: slice >> gsh (the group size is a power of two >= 16,
  // checked on the host)
  const int gsh = __ffs(ent->group_size) - 1 - 4;
  const int n_groups = K >> (gsh + 4);

  // loads of stage kb into its ring slot (one thread)
  auto issue_stage = [&](int kb) {
    const int s = kb % STAGES;
    uint8_t* stage = smem + s * S::kStageBytes;
    mbar_arrive_expect_tx(&full[s], uint32_t(S::kTokBytes + NB * S::kBoxBytes));
    tma_load_2d(stage, &tmap_a, &full[s], kb * kBK, row0);
    const uint64_t stream_once = policy_evict_first();
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const int mb = kGLU ? (b < NB / 2 ? 0 : 1) : mat;
      const int c0 = kGLU ? f0 + 64 * (b % (NB / 2)) : f0 + 64 * b;  // first column of the box
      tma_load_2d_hint(stage + S::offW + b * S::kBoxBytes, &ent->qw8[mb], &full[s], c0 / 8,
                       kb * kBK, stream_once);
    }
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      done[i] = 0;
    }
    *s_abort = 0;
    fence_mbarrier_init();
    tma_prefetch_desc(&tmap_a);
  }
  if (lane == 0) {
    // any warp may issue loads (as a refiller); the descriptors were written to
    // global memory by a copy before the launch
    for (int m2 = 0; m2 < 3; ++m2) {
      if (!(ent->present & (1 << m2))) continue;
      tensormap_acquire(&ent->qw8[m2]);
    }
  }
  if (threadIdx.x == 0) {
    const int first = KB < STAGES ? KB : STAGES;
    for (int kb = 0; kb < first; ++kb) issue_stage(kb);
    *s_issued = first;
  }
  __syncthreads();

  // ------------------------------------------------------------------ consumers
  const int box = warp % NB, kq = warp / NB;
  const int g = lane >> 2, t = lane & 3;
  const int mb = kGLU ? (box < NB / 2 ? 0 : 1) : mat;
  const int J = kGLU ? (f0 + 64 * (box % (NB / 2))) / 8 + g : (f0 + 64 * box) / 8 + g;
  const bool jvalid = 8 * J < N;
  const int nt_used = (rows_valid + 7) >> 3;
  const __half* scol = ent->scales[mb] + 8 * size_t(J);
  const int32_t* zcol = ent->zeros[mb] + J;

  float acc[4][NT][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[i][n][c] = 0.f;

  // shared-memory offsets within a stage, fixed for the whole loop: the lane's
  // weight words (rows 2t, 2t+1, 2t+8, 2t+9, column g of its box) of slice j,
  // and its ldmatrix row address (token row (lane & 7) + 8 (lane >> 4) of n
  // tile pair p, 16-byte chunk (lane >> 3) & 1 of the slice, 128-byte swizzle)
  constexpr int JS = 4 / KSPLIT, NP = (NT + 1) / 2;
  uint32_t w_off[JS], b_off[JS][NP];
#pragma unroll
  for (int j = 0; j < JS; ++j) {
    const int q = kq + KSPLIT * j;
    w_off[j] = S::offW + box * S::kBoxBytes + ((16 * q + 2 * t) * 8 + g) * 4;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      // an odd last n tile takes ldmatrix.x2, whose addresses come from lanes
      // 0-15: keep the other lanes' (unused) rows inside the box too
      const int r = 16 * p + (2 * p + 1 < NT ? (lane & 7) + 8 * (lane >> 4) : (lane & 7));
      b_off[j][p] = r * 128 + ((((2 * q + ((lane >> 3) & 1)) ^ (r & 7))) << 4);
    }
  }

  // scale / zero words of a group (zero for feature columns past N)
  auto load_params = [&](int grp, uint4& sc, uint32_t& zw) {
    sc = make_uint4(0, 0, 0, 0);
    zw = 0;
    if (jvalid) {
      sc = __ldg(reinterpret_cast<const uint4*>(scol + size_t(grp) * N));
      zw = uint32_t(__ldg(zcol + size_t(grp) * (N / 8)));
    }
  };
  // the first group after `grp` that one of this warp's slices falls in
  auto next_group = [&](int grp) {
    const int b = (grp + 1) << gsh;  // first slice of the following group
    return (b + ((kq - b) & (KSPLIT - 1))) >> gsh;
  };
  SkParams P;
  int cur_group = kq >> gsh;
  {
    uint4 sc;
    uint32_t zw;
    load_params(cur_group, sc, zw);
    sk_params(zw, sc, P);
  }
  int nx_group = next_group(cur_group);
  uint4 nx_sc = make_uint4(0, 0, 0, 0);
  uint32_t nx_zw = 0;
  if (nx_group < n_groups) load_params(nx_group, nx_sc, nx_zw);

  // one 16-deep slice with NTU live token tiles
  auto slice = [&](auto ntu_c, uint32_t base, int j) {
    constexpr int NTU = decltype(ntu_c)::value;
    const uint32_t wr = base + w_off[j];
    const uint32_t w0 = lds32(wr), w1 = lds32(wr + 32), w2 = lds32(wr + 256),
                   w3 = lds32(wr + 288);
    uint32_t b[NT][2];
#pragma unroll
    for (int n = 0; n < NTU; n += 2) {
      if (n + 1 < NTU) ldmatrix_x4(base + b_off[j][n / 2], b[n][0], b[n][1], b[n + 1][0],
                                   b[n + 1][1]);
      else ldmatrix_x2(base + b_off[j][n / 2], b[n][0], b[n][1]);
    }
    uint32_t lo0[4], hi0[4], lo8[4], hi8[4];
    sk_deq4(prmt(w0, w1, 0x5410), P, 0, lo0);  // features 0-3, k 2t / 2t+1
    sk_deq4(prmt(w0, w1, 0x7632), P, 4, hi0);  // features 4-7
    sk_deq4(prmt(w2, w3, 0x5410), P, 0, lo8);  // features 0-3, k 2t+8 / 2t+9
    sk_deq4(prmt(w2, w3, 0x7632), P, 4, hi8);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t a[4] = {lo0[i], hi0[i], lo8[i], hi8[i]};
#pragma unroll
      for (int n = 0; n < NTU; ++n) mma_16816(acc[i][n], a, b[n][0], b[n][1]);
    }
  };

  // group switch: the scale / zero words of the next group were requested a
  // group ago (clamped for a K tail past the last group; those rows hold zero
  // tokens)
  auto enter_group = [&](int grp) {
    grp = grp < n_groups ? grp : n_groups - 1;
    if (grp == cur_group) return;
    if (grp != nx_group) load_params(grp, nx_sc, nx_zw);
    sk_params(nx_zw, nx_sc, P);
    cur_group = grp;
    nx_group = next_group(grp);
    if (nx_group < n_groups) load_params(nx_group, nx_sc, nx_zw);
  };

  bool ok = true;
  int kb = 0;
  // The k loop, specialised on the live token tiles (fixed for the CTA) and on
  // whether a stage lies in one group (group size >= 64), so that a stage's
  // slices are straight-line code the compiler can interleave.
  auto main_loop = [&](auto ntu_c, auto one_group_c) {
    constexpr bool kOneGroup = decltype(one_group_c)::value;
    for (; kb < KB; ++kb) {
      const int s = kb % STAGES;
      if (!wait_any(&full[s], (kb / STAGES) & 1, s_abort, err)) {
        ok = false;
        break;
      }
      const uint32_t base = smem_u32(smem + s * S::kStageBytes);
      if (kOneGroup) enter_group((4 * kb) >> gsh);
#pragma unroll
      for (int j = 0; j < JS; ++j) {
        if (!kOneGroup) enter_group((4 * kb + kq + KSPLIT * j) >> gsh);
        slice(ntu_c, base, j);
      }
      // the last warp done with this slot refills it with the stage STAGES ahead
      __syncwarp();
      if (lane == 0) {
        if (atom_add_acq_rel(&done[s], 1u) == uint32_t(S::kConsumers - 1)) {
          done[s] = 0;
          if (kb + STAGES < KB) {
            fence_proxy_async_smem();
            issue_stage(kb + STAGES);
            atomicMax(s_issued, kb + STAGES + 1);
          }
        }
      }
    }
  };
  auto run = [&](auto ntu_c) {
    if (gsh >= 2) main_loop(ntu_c, std::true_type{});
    else main_loop(ntu_c, std::false_type{});
  };
  if (nt_used >= NT) run(std::integral_constant<int, NT>{});
  else if (NT > 1 && nt_used == 1) run(std::integral_constant<int, 1>{});
  else if (NT > 2 && nt_used == 2) run(std::integral_constant<int, (NT > 2 ? 2 : 1)>{});
  else run(std::integral_constant<int, (NT > 3 ? 3 : 1)>{});
  if (!ok && lane == 0) {
    // a wait ran out: let the copies in flight on this warp's slots land before exit
    const int last = *reinterpret_cast<volatile int*>(s_issued);
    for (int i = kb; i < last && i < kb + STAGES; ++i) wait_drain(&full[i % STAGES], (i / STAGES) & 1);
  }

  // ---------------------------------------------------------------- epilogue
  constexpr int kCons = S::kThreads;
  if (bar_any(1, kCons, !ok)) return;  // a wait ran out: write nothing
  float* red = reinterpret_cast<float*>(smem);  // the ring is free: every stage consumed
  constexpr int kAcc = S::kAcc;
  auto slot_ptr = [&](int slot, int i) { return red + (size_t(slot) * kAcc + i) * 32 + lane; };
  if (KSPLIT > 1) {
    if (kq > 0) {
      int i = 0;
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int c = 0; c < 4; ++c, ++i) *slot_ptr((kq - 1) * NB + box, i) = acc[a][n][c];
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kCons) : "memory");
    if (kq == 0) {
      for (int j = 1; j < KSPLIT; ++j) {
        int i = 0;
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int c = 0; c < 4; ++c, ++i) acc[a][n][c] += *slot_ptr((j - 1) * NB + box, i);
      }
    }
  }
  if (kGLU) {
    // the up boxes hand their sums to the gate boxes of the same features
    if (KSPLIT > 1) asm volatile("bar.sync 1, %0;" ::"r"(kCons) : "memory");
    if (kq == 0 && box >= NB / 2) {
      int i = 0;
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int c = 0; c < 4; ++c, ++i) *slot_ptr(box - NB / 2, i) = acc[a][n][c];
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kCons) : "memory");
    if (kq != 0 || box >= NB / 2) return;
    int i = 0;
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int c = 0; c < 4; ++c, ++i)
          acc[a][n][c] = silu_f32(acc[a][n][c]) * *slot_ptr(box, i);
  } else {
    if (kq != 0) return;
    if (MODE == LR_FFN_MODE_SILU) {
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[a][n][c] = silu_f32(acc[a][n][c]);
    }
  }
  if (!jvalid) return;
  // lane holds features 8J..8J+7 of tokens 8n + 2t (c = 0, 2) and 8n + 2t + 1 (c = 1, 3)
#pragma unroll
  for (int n = 0; n < NT; ++n) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = 8 * n + 2 * t + h;
      if (r < rows_valid) {
        uint4 o;
        __half2* p = reinterpret_cast<__half2*>(&o);
        p[0] = __floats2half2_rn(acc[0][n][h], acc[1][n][h]);
        p[1] = __floats2half2_rn(acc[2][n][h], acc[3][n][h]);
        p[2] = __floats2half2_rn(acc[0][n][2 + h], acc[1][n][2 + h]);
        p[3] = __floats2half2_rn(acc[2][n][2 + h], acc[3][n][2 + h]);
        *reinterpret_cast<uint4*>(C + size_t(row0 + r) * N + 8 * size_t(J)) = o;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <class S, int MODE>
static int launch_skinny_shape(const void* A, int K, int R, const ExpertEntry* table, int E,
                               int mat, int N, const int32_t* seg_start, const int32_t* seg_len,
                               int max_rows, __half* C, int32_t* err, cudaStream_t stream) {
  auto kern = w4a16_skinny_kernel<S, MODE>;
  static unsigned long long configured = 0;
  if (const int rc = set_dyn_smem_once(kern, S::kTotal, configured, true)) return rc;
  CUtensorMap ta;
  if (const int rc = encode_rows_cached(&ta, A, K, R, uint32_t(S::TR), CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  constexpr int BO = MODE == LR_FFN_MODE_SWIGLU ? S::NB * 32 : S::NB * 64;
  const int n_slabs = (N + BO - 1) / BO;
  const int m_tiles = (max_rows + S::TR - 1) / S::TR;
  const long grid = long(E) * m_tiles * n_slabs;
  if (grid > 0x7fffffffL) return LR_ERR_UNSUPPORTED;
  kern<<<unsigned(grid), S::kThreads, S::kTotal, stream>>>(ta, table, E, mat, K, N, seg_start,
                                                           seg_len, max_rows, R, n_slabs,
                                                           m_tiles, C, err);
  LR_LAUNCH_CHECK();
  return LR_OK;
}

// SwiGLU (gate/up): 4 boxes = 128 features x (gate, up) per unit, two warps per
// box.  Plain / SiLU (down, PR1 up): 2 boxes = 128 features, four warps per box.
template <int MODE, int TR>
static int launch_skinny_tr(const void* A, int K, int R, const ExpertEntry* t, int E, int mat,
                            int N, const int32_t* ss, const int32_t* sl, int mr, __half* C,
                            int32_t* err, cudaStream_t st) {
  if (MODE == LR_FFN_MODE_SWIGLU)
    return launch_skinny_shape<SkinnyShape<4, 2, TR, 6>, MODE>(A, K, R, t, E, mat, N, ss, sl, mr,
                                                               C, err, st);
  return launch_skinny_shape<SkinnyShape<2, 4, TR, 9>, MODE>(A, K, R, t, E, mat, N, ss, sl, mr, C,
                                                             err, st);
}

template <int MODE>
int launch_skinny(const void* A, int K, int R, const ExpertEntry* t, int E, int mat, int N,
                  const int32_t* ss, const int32_t* sl, int mr, __half* C, int32_t* err,
                  cudaStream_t st) {
  if (mr <= 16) return launch_skinny_tr<MODE, 16>(A, K, R, t, E, mat, N, ss, sl, mr, C, err, st);
  if (mr <= 24) return launch_skinny_tr<MODE, 24>(A, K, R, t, E, mat, N, ss, sl, mr, C, err, st);
  return launch_skinny_tr<MODE, 32>(A, K, R, t, E, mat, N, ss, sl, mr, C, err, st);
}

template int launch_skinny<LR_FFN_MODE_PLAIN>(const void*, int, int, const ExpertEntry*, int, int,
                                              int, const int32_t*, const int32_t*, int, __half*,
                                              int32_t*, cudaStream_t);
template int launch_skinny<LR_FFN_MODE_SILU>(const void*, int, int, const ExpertEntry*, int, int,
                                             int, const int32_t*, const int32_t*, int, __half*,
                                             int32_t*, cudaStream_t);
template int launch_skinny<LR_FFN_MODE_SWIGLU>(const void*, int, int, const ExpertEntry*, int,
                                               int, int, const int32_t*, const int32_t*, int,
                                               __half*, int32_t*, cudaStream_t);

}  // namespace lr
