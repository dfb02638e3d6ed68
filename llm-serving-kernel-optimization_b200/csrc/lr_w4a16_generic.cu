// lr_w4a16_generic.cu -- grouped W4A16 GEMM for the shapes the tensor-memory
// (TMA-fed) kernels do not take.
//
// The packed format admits any N % 8 == 0 and any group size dividing K
// (reference lightning_router/quantization/pack_weights.py:44-45), and the
// reference's quantized_matmul masks any M and N
// (lightning_router/kernels/quantized_matmul.py:122-173).  The tcgen05 kernel
// needs K % 64, group % 64 and N % 32; the mma.sync kernel needs K % 8, a
// power-of-two group >= 16 and N % 32 (TMA strides).  Everything else -- N = 48,
// K = 40, a group of 8, an fp16 A whose rows are not 16-byte aligned -- runs
// here: one thread per (row, 8 output features), the weights dequantized with
// the reference's single rounding fp16(scale * (q - zero)) and accumulated in
// fp32 in k order.  It is a correctness path for odd shapes, not a fast one.
#include "lr_w4a16.cuh"

namespace lr {

constexpr int kGenThreads = 128;

// out[i] = fp16(scale_i * (q_i - z_i)) as fp32, features 8J .. 8J+7 of one k row.
LR_DEVICE void deq8_f32(uint32_t w, uint32_t zw, const uint4& sc, float (&out)[8]) {
  const __half* s = reinterpret_cast<const __half*>(&sc);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = int((w >> (4 * i)) & 15u) - int((zw >> (4 * i)) & 15u);
    out[i] = __half2float(__hmul(s[i], __int2half_rn(d)));
  }
}

template <int MODE>
__global__ void __launch_bounds__(kGenThreads)
    w4a16_generic_kernel(const ExpertEntry* __restrict__ table, int E, int mat, int K, int N,
                         int gs, const int32_t* __restrict__ seg_start,
                         const int32_t* __restrict__ seg_len, int max_rows, int R,
                         const __half* __restrict__ A, __half* __restrict__ C, int32_t* err) {
  constexpr bool kGLU = MODE == LR_FFN_MODE_SWIGLU;
  const int nwords = N / 8;
  const int J = blockIdx.x * kGenThreads + threadIdx.x;  // word column: features 8J .. 8J+7
  const long rows_total = long(E) * max_rows;
  for (long u = blockIdx.y; u < rows_total; u += gridDim.y) {
    const int e = int(u / max_rows), r = int(u % max_rows);
    int st = seg_start ? __ldg(seg_start + e) : 0;
    int len = seg_start ? __ldg(seg_len + e) : R;
    const bool reporter = r == 0 && blockIdx.x == 0 && threadIdx.x == 0;
    if (len < 0) len = 0;
    if (len > max_rows) {
      if (reporter) report(err, LR_DEVERR_BAD_SEGMENT);
      len = max_rows;
    }
    if (st < 0 || st + len > R) {
      if (reporter) report(err, LR_DEVERR_BAD_SEGMENT);
      continue;
    }
    if (r >= len || J >= nwords) continue;
    const int row = st + r;
    const ExpertEntry* ent = table + e;
    const __half* x = A + size_t(row) * K;
    const int m0 = kGLU ? 0 : mat;
    const int32_t* q0 = ent->qw[m0] + J;
    const int32_t* q1 = kGLU ? ent->qw[1] + J : q0;
    float acc0[8], acc1[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc0[i] = acc1[i] = 0.f;
    for (int gi = 0; gi < K / gs; ++gi) {
      const uint4 sc0 = __ldg(reinterpret_cast<const uint4*>(ent->scales[m0] + size_t(gi) * N + 8 * J));
      const uint32_t zw0 = uint32_t(__ldg(ent->zeros[m0] + size_t(gi) * nwords + J));
      uint4 sc1 = sc0;
      uint32_t zw1 = zw0;
      if (kGLU) {
        sc1 = __ldg(reinterpret_cast<const uint4*>(ent->scales[1] + size_t(gi) * N + 8 * J));
        zw1 = uint32_t(__ldg(ent->zeros[1] + size_t(gi) * nwords + J));
      }
      for (int k = gi * gs; k < (gi + 1) * gs; ++k) {
        const float xv = __half2float(x[k]);
        float w[8];
        deq8_f32(uint32_t(__ldg(q0 + size_t(k) * nwords)), zw0, sc0, w);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc0[i] = fmaf(xv, w[i], acc0[i]);
        if (kGLU) {
          deq8_f32(uint32_t(__ldg(q1 + size_t(k) * nwords)), zw1, sc1, w);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc1[i] = fmaf(xv, w[i], acc1[i]);
        }
      }
    }
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (kGLU) o[i] = silu_f32(acc0[i]) * acc1[i];
      else if (MODE == LR_FFN_MODE_SILU) o[i] = silu_f32(acc0[i]);
      else o[i] = acc0[i];
    }
    *reinterpret_cast<uint4*>(C + size_t(row) * N + 8 * size_t(J)) = pack_half8(o);
  }
}

template <int MODE>
int launch_generic(const void* A, int K, int R, const ExpertEntry* table, int E, int mat, int N,
                   int group_size, const int32_t* seg_start, const int32_t* seg_len,
                   int max_rows, __half* C, int32_t* err, cudaStream_t stream) {
  const int nwords = N / 8;
  const long rows = long(E) * max_rows;
  dim3 grid(unsigned((nwords + kGenThreads - 1) / kGenThreads),
            unsigned(rows < 65535 ? rows : 65535));
  w4a16_generic_kernel<MODE><<<grid, kGenThreads, 0, stream>>>(
      table, E, mat, K, N, group_size, seg_start, seg_len, max_rows, R,
      static_cast<const __half*>(A), C, err);
  LR_LAUNCH_CHECK();
  return LR_OK;
}

template int launch_generic<LR_FFN_MODE_PLAIN>(const void*, int, int, const ExpertEntry*, int,
                                               int, int, int, const int32_t*, const int32_t*,
                                               int, __half*, int32_t*, cudaStream_t);
template int launch_generic<LR_FFN_MODE_SILU>(const void*, int, int, const ExpertEntry*, int, int,
                                              int, int, const int32_t*, const int32_t*, int,
                                              __half*, int32_t*, cudaStream_t);
template int launch_generic<LR_FFN_MODE_SWIGLU>(const void*, int, int, const ExpertEntry*, int,
                                                int, int, int, const int32_t*, const int32_t*,
                                                int, __half*, int32_t*, cudaStream_t);

}  // namespace lr
