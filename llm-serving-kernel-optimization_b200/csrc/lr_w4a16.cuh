// lr_w4a16.cuh -- pieces shared by the W4A16 expert GEMM kernels: the per-expert
// weight table, int4 -> fp16 dequantization helpers, bounded pipeline waits and
// tensor-map encoding.
#pragma once
#include <cudaTypedefs.h>

#include "lr_common.cuh"

namespace lr {

// ---------------------------------------------------------------------------
// per-expert weight table (device resident, written once per weight set)
// ---------------------------------------------------------------------------
struct alignas(128) ExpertEntry {
  CUtensorMap qw32[3];  // packed weights, box {32 words = 256 features, 64 rows}
  CUtensorMap qw16[3];  // packed weights, box {16 words = 128 features, 64 rows}
  CUtensorMap qw8[3];   // packed weights, box {8 words = 64 features, 64 rows}
  const int32_t* qw[3];
  const __half* scales[3];
  const int32_t* zeros[3];
  int32_t K[3];
  int32_t N[3];
  int32_t group_size;
  int32_t present;  // bit m set when matrix m is encoded
  int32_t tma;      // bit m set when matrix m's tensor maps are encoded (N % 32 == 0)
};
static_assert(sizeof(ExpertEntry) % 128 == 0, "table entry alignment");

constexpr int kBK = 64;       // k per pipeline step
constexpr int kMaxGemmExperts = 256;
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s
constexpr uint64_t kDrainLimitNs = 100000000ull;  // 100 ms

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
// order (a permutation of the tile's N columns) and the epilogue puts each
// group of eight accumulator columns back into feature order.
LR_DEVICE uint4 deq_word(uint32_t w, const DeqParams& P) {
  uint4 o;
  o.x = h2_mul(h2_sub(nib_pair(w, 0), P.z[0]), P.s[0]);
  o.y = h2_mul(h2_sub(nib_pair(w, 1), P.z[1]), P.s[1]);
  o.z = h2_mul(h2_sub(nib_pair(w, 2), P.z[2]), P.s[2]);
  o.w = h2_mul(h2_sub(nib_pair(w, 3), P.z[3]), P.s[3]);
  return o;
}

// Eight accumulator columns in the operand's order (f0 f4 f1 f5 f2 f6 f3 f7)
// -> eight fp16 features in order.
LR_DEVICE uint4 pack8_feature_order(const float* v) {
  uint4 o;
  __half2* h = reinterpret_cast<__half2*>(&o);
  h[0] = __floats2half2_rn(v[0], v[2]);  // f0 f1
  h[1] = __floats2half2_rn(v[4], v[6]);  // f2 f3
  h[2] = __floats2half2_rn(v[1], v[3]);  // f4 f5
  h[3] = __floats2half2_rn(v[5], v[7]);  // f6 f7
  return o;
}

// Named barrier over the 128 threads of one epilogue group that also returns
// whether any of them passed `pred`.
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
// host side
// ---------------------------------------------------------------------------
inline PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
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

inline int encode_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t dim0,
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

// SM count of the current device (queried once per device ordinal below 64).
inline int current_sm_count(int* out) {
  static int cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return LR_ERR_NO_DEVICE;
  if (dev < 64 && __atomic_load_n(&cache[dev], __ATOMIC_RELAXED) > 0) {
    *out = cache[dev];
    return LR_OK;
  }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
    return LR_ERR_NO_DEVICE;
  if (dev < 64) __atomic_store_n(&cache[dev], sms, __ATOMIC_RELAXED);
  *out = sms;
  return LR_OK;
}

// Tensor map of a row-major fp16 operand (K columns, R rows, box of 64 x
// box_rows), reused while the same host thread passes the same operand: a
// small per-thread cache keyed by device, address, shape, box and swizzle.
inline int encode_rows_cached(CUtensorMap* out, const void* A, int K, int R, uint32_t box_rows,
                              CUtensorMapSwizzle sw) {
  struct Entry {
    const void* a;
    int K, R, dev;
    uint32_t box;
    int sw;
    CUtensorMap map;
  };
  thread_local Entry cache[8];
  thread_local int used = 0, next = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return LR_ERR_NO_DEVICE;
  for (int i = 0; i < used; ++i) {
    const Entry& c = cache[i];
    if (c.a == A && c.K == K && c.R == R && c.dev == dev && c.box == box_rows && c.sw == int(sw)) {
      *out = c.map;
      return LR_OK;
    }
  }
  const int rc = encode_2d(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, A, uint64_t(K), uint64_t(R),
                           uint64_t(K) * 2, kBK, box_rows, sw);
  if (rc) return rc;
  cache[next] = Entry{A, K, R, dev, box_rows, int(sw), *out};
  next = (next + 1) % 8;
  if (used < 8) ++used;
  return LR_OK;
}

// Grouped GEMM for expert segments of at most kSkinnyMaxRows rows (decode):
// mma.sync with the weights as the M operand (lr_w4a16_skinny.cu).  Needs
// K % 8 == 0 (16-byte token rows for TMA) and a group size that is a power of
// two >= 16.
constexpr int kSkinnyMaxRows = 32;
// Grouped GEMM for any shape of the packed format (lr_w4a16_generic.cu): CUDA
// cores, for what neither TMA-fed kernel takes.
template <int MODE>
int launch_generic(const void* A, int K, int R, const ExpertEntry* table, int E, int mat, int N,
                   int group_size, const int32_t* seg_start, const int32_t* seg_len,
                   int max_rows, __half* C, int32_t* err, cudaStream_t stream);
// Grouped GEMM for expert segments of at most 32 rows on 8-bit tcgen05 operands
// (lr_w4a16_i8.cu): INT4 codes as unsigned bytes, token rows as two signed
// 8-bit terms per 128-k block, group scale and zero folded per block.  Needs
// K % 128 == 0, group_size % 128 == 0, N % 32 == 0 and a workspace of
// i8_workspace_bytes(R, K) bytes (128-byte aligned) for the token terms.
bool i8_eligible(int K, int N, int group_size, int max_rows);
size_t i8_workspace_bytes(int R, int K);
template <int MODE>
int launch_i8(const void* A, int K, int R, const ExpertEntry* table, int E, int mat, int N,
              int group_size, const int32_t* seg_start, const int32_t* seg_len, int max_rows,
              __half* C, void* ws, int32_t* err, cudaStream_t stream);
template <int MODE>
int launch_skinny(const void* A, int K, int R, const ExpertEntry* table, int E, int mat, int N,
                  const int32_t* seg_start, const int32_t* seg_len, int max_rows, __half* C,
                  int32_t* err, cudaStream_t stream);

}  // namespace lr

namespace lr {

// ---------------------------------------------------------------------------
// persistent tile schedule shared by the grouped kernels
// ---------------------------------------------------------------------------
// One warp reads the E row segments (clamping and flagging bad ones) and writes
// per expert: first tile index (tbase, E+1 entries, tbase[E] = total), segment
// start and length, and the number of token tiles (rows / ROWS rounded up).
// Tiles of an expert are numbered token tile fastest, then feature tile.
LR_DEVICE void build_tile_table(const int32_t* __restrict__ seg_start,
                                const int32_t* __restrict__ seg_len, int E, int R, int max_rows,
                                int rows_per_tile, int n_tiles, int* s_tbase, int* s_start,
                                int* s_len, int* s_mt, int32_t* err) {
  const int lane = threadIdx.x & 31;
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
    const int mt = (len + rows_per_tile - 1) / rows_per_tile;
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

// tile -> (expert, token tile, feature tile).  Within an expert the token tiles
// vary fastest (CTAs running at the same time share weight columns through L2),
// or, with n_fastest, the feature tiles (they share token rows instead: better
// when the expert's token rows outweigh its weights, e.g. a long-K down
// projection).
LR_DEVICE void decode_tile(const int* s_tbase, const int* s_mt, int E, int tile, int& e, int& mt,
                           int& nt, bool n_fastest = false, int n_tiles = 1) {
  int lo = 0, hi = E;  // last e with s_tbase[e] <= tile
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (s_tbase[mid] <= tile) lo = mid;
    else hi = mid;
  }
  e = lo;
  const int local = tile - s_tbase[e];
  if (n_fastest) {
    mt = local / n_tiles;
    nt = local - mt * n_tiles;
  } else {
    nt = local / s_mt[e];
    mt = local - nt * s_mt[e];
  }
}

}  // namespace lr
