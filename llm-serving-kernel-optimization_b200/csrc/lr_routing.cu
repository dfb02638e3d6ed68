// lr_routing.cu -- gating, dispatch and combine kernels of the MoE layer (sm_100a).
//
// Data layout (S = T*k slots, slot s = t*k + j):
//   expert_ids[S], gate_weights[S]              per slot
//   offsets[E+1]                                uncapped CSR over experts
//   rows [offsets[e], offsets[e+1])             expert e; the first min(count, C)
//                                               rows are its kept slots in slot order
//   permuted[S][d], routing_w[S], source_idx[S] per row
//   slot_pos[S]                                 row of each slot, -1 if dropped
//
// Dispatch is two launches:
//   route   : per block of slots, top-k (or given ids), per-slot rank inside the
//             block for its expert (warp match + per-warp counts in shared
//             memory), per-block histogram; the last block to finish scans the
//             (block x expert) histogram into per-block bases and the CSR offsets.
//   permute : each slot's row = offsets[e] + base[block][e] + rank; kept iff the
//             expert-wide rank < capacity.  Token rows are copied with 128-bit
//             vector loads/stores; for gated routing each token row is read once
//             and written to its k rows.
// Small batches (T <= 256, decode) take the gate projection into the route
// launch (gate_route_small_kernel) and copy the rows in a second one.
#include "lr_common.cuh"

namespace lr {

constexpr int kRouteThreads = 256;   // tokens per block of the gating route kernel
constexpr int kSlotBlock = 1024;     // slots per block of the given-ids route kernel
constexpr int kWarps = kRouteThreads / 32;

// ---------------------------------------------------------------------------
// workspace layout
// ---------------------------------------------------------------------------
struct RouteWs {
  int32_t* ticket;
  int32_t* blk_counts;  // [B][E]
  int32_t* blk_base;    // [B][E]
  double* blk_psum;     // [B][E] (gating route only)
};

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

static size_t route_ws_bytes_for(int B, int E, bool psum) {
  size_t b = 256;
  b += align256(size_t(B) * E * sizeof(int32_t));
  b += align256(size_t(B) * E * sizeof(int32_t));
  if (psum) b += align256(size_t(B) * E * sizeof(double));
  return b;
}

static RouteWs carve_route_ws(void* ws, int B, int E, bool psum) {
  char* p = static_cast<char*>(ws);
  RouteWs r;
  r.ticket = reinterpret_cast<int32_t*>(p);
  p += 256;
  r.blk_counts = reinterpret_cast<int32_t*>(p);
  p += align256(size_t(B) * E * sizeof(int32_t));
  r.blk_base = reinterpret_cast<int32_t*>(p);
  p += align256(size_t(B) * E * sizeof(int32_t));
  r.blk_psum = psum ? reinterpret_cast<double*>(p) : nullptr;
  return r;
}

// ---------------------------------------------------------------------------
// gate projection: logits[T,E] = h[T,d] . wg[E,d]^T (+bias), fp32 accumulate.
// One warp per (16-token tile, 32-expert group); mma.sync m16n8k16 fragments
// loaded straight from global (rows are read once per expert group).
// ---------------------------------------------------------------------------
LR_DEVICE uint32_t ld_u32(const __half* p) { return __ldg(reinterpret_cast<const uint32_t*>(p)); }

LR_DEVICE void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// One block per (16-token tile, 32-expert group).  Its 8 warps split d into
// 8 contiguous chunks (each a multiple of 16), accumulate 16x32 partial logits
// with mma.sync, and the partials are summed in warp order through shared
// memory (deterministic), so small token counts still spread over many warps.
constexpr int kGateWarps = 8;

__global__ void __launch_bounds__(kGateWarps * 32)
    gate_logits_kernel(const __half* __restrict__ h, const __half* __restrict__ wg,
                       const float* __restrict__ bias, int T, int d, int E, int n_egroups,
                       float* __restrict__ logits) {
  __shared__ float red[kGateWarps][16][33];
  const int tile = blockIdx.x / n_egroups;
  const int eg = blockIdx.x % n_egroups;
  const int t0 = tile * 16;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int e0 = eg * 32;
  const int row0 = t0 + g, row1 = t0 + g + 8;
  const bool r0 = row0 < T, r1 = row1 < T;
  const int kc = ((d / 16 + kGateWarps - 1) / kGateWarps) * 16;
  const int kbeg = warp * kc, kend = min(d, kbeg + kc);
  const __half* h0 = h + size_t(r0 ? row0 : 0) * d + 2 * tq;
  const __half* h1 = h + size_t(r1 ? row1 : 0) * d + 2 * tq;
  const __half* wrow[4];
  bool wok[4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int e = e0 + nt * 8 + g;
    wok[nt] = e < E;
    wrow[nt] = wg + size_t(wok[nt] ? e : 0) * d + 2 * tq;
  }
  float acc[4][4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[nt][i] = 0.f;

#pragma unroll 2
  for (int k0 = kbeg; k0 < kend; k0 += 16) {
    uint32_t a[4];
    a[0] = r0 ? ld_u32(h0 + k0) : 0u;
    a[1] = r1 ? ld_u32(h1 + k0) : 0u;
    a[2] = r0 ? ld_u32(h0 + k0 + 8) : 0u;
    a[3] = r1 ? ld_u32(h1 + k0 + 8) : 0u;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      if (e0 + nt * 8 < E) {  // warp-uniform
        const uint32_t b0 = wok[nt] ? ld_u32(wrow[nt] + k0) : 0u;
        const uint32_t b1 = wok[nt] ? ld_u32(wrow[nt] + k0 + 8) : 0u;
        mma_16816(acc[nt], a, b0, b1);
      }
    }
  }
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) red[warp][(i < 2) ? g : g + 8][nt * 8 + 2 * tq + (i & 1)] = acc[nt][i];
  __syncthreads();
  for (int o = threadIdx.x; o < 16 * 32; o += kGateWarps * 32) {
    const int rr = o >> 5, cc = o & 31;
    const int row = t0 + rr, col = e0 + cc;
    if (row < T && col < E) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kGateWarps; ++w) v += red[w][rr][cc];
      if (bias) v += bias[col];
      logits[size_t(row) * E + col] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// block-level slot ranking (shared by both route kernels)
// ---------------------------------------------------------------------------
// Ranks one chunk of <= 256 consecutive slots (thread tid owns slot `valid ? e : -1`).
// s_wcnt[warp][e] receives per-warp counts (one write per (warp, expert) by the
// warp's leader for that expert), then is turned into exclusive prefixes that
// start from the running per-expert count s_run[e].  Returns the block-local
// rank of the thread's slot among slots of the same expert (slot order).
LR_DEVICE int rank_chunk(int e, bool valid, int E, int32_t* s_wcnt, int32_t* s_run) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < kWarps * E; i += kRouteThreads) s_wcnt[i] = 0;
  __syncthreads();
  const unsigned peers = __match_any_sync(0xffffffffu, valid ? e : -1);
  const int lrank = __popc(peers & lanemask_lt());
  if (valid && (__ffs(peers) - 1) == lane) s_wcnt[warp * E + e] = __popc(peers);
  __syncthreads();
  for (int x = tid; x < E; x += kRouteThreads) {
    int run = s_run[x];
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const int c = s_wcnt[w * E + x];
      s_wcnt[w * E + x] = run;
      run += c;
    }
    s_run[x] = run;
  }
  __syncthreads();
  const int r = valid ? s_wcnt[warp * E + e] + lrank : -1;
  __syncthreads();
  return r;
}

// Last-block tail: scans blk_counts over blocks per expert into blk_base,
// writes offsets / kept_counts and the aux loss, resets the ticket.
LR_DEVICE void route_tail(const RouteWs& ws, int B, int E, int C, int num_slots, int T, int k,
                          float lbw, int32_t* offsets, int32_t* kept_counts, float* aux_loss,
                          double* prob_sums, int32_t* s_tot, double* s_P) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = warp; e < E; e += kWarps) {
    int carry = 0;
    double psum = 0.0;
    for (int b0 = 0; b0 < B; b0 += 32) {
      const int b = b0 + lane;
      const int v = (b < B) ? __ldcg(ws.blk_counts + size_t(b) * E + e) : 0;
      if (ws.blk_psum && b < B) psum += __ldcg(ws.blk_psum + size_t(b) * E + e);
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      if (b < B) ws.blk_base[size_t(b) * E + e] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
    if (lane == 0) {
      s_tot[e] = carry;
      s_P[e] = psum;
    }
  }
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    double aux = 0.0;
    offsets[0] = 0;
    for (int e = 0; e < E; ++e) {
      run += s_tot[e];
      offsets[e + 1] = run;
      if (kept_counts) kept_counts[e] = min(s_tot[e], C);
      if (prob_sums) prob_sums[e] = s_P[e];
      aux += (double(s_tot[e]) / double(num_slots)) * (s_P[e] / double(T));
    }
    if (aux_loss) aux_loss[0] = static_cast<float>(double(lbw) * double(E) * aux);
    *ws.ticket = 0;
    (void)k;
  }
}

LR_DEVICE bool arrive_last(int32_t* ticket, int num_blocks, int* s_flag) {
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int t = atomicAdd(ticket, 1);
    *s_flag = (t == num_blocks - 1);
  }
  __syncthreads();
  if (*s_flag) __threadfence();
  return *s_flag != 0;
}

// ---------------------------------------------------------------------------
// gating route: top-k softmax per token + slot ranks + histogram (+aux sums)
// ---------------------------------------------------------------------------
// One token's fp32 logits -> softmax probabilities p, the k experts with the
// largest logits (descending, lowest index first on ties) and their weights
// p / (sum of the selected p + 1e-9) (reference gating.py:69-85).
template <int MAXE>
LR_DEVICE void topk_softmax(const float (&l)[MAXE], int E, int k, float (&p)[MAXE],
                            int (&ids)[kMaxTopK], float (&wsel)[kMaxTopK]) {
  float m = l[0];
#pragma unroll
  for (int i = 1; i < MAXE; ++i)
    if (i < E) m = fmaxf(m, l[i]);
  float z = 0.f;
#pragma unroll
  for (int i = 0; i < MAXE; ++i) {
    p[i] = (i < E) ? expf(l[i] - m) : 0.f;
    z += p[i];
  }
#pragma unroll
  for (int i = 0; i < MAXE; ++i) p[i] = (i < E) ? p[i] / z : 0.f;

  uint64_t sel = 0;
  float psel[kMaxTopK];
  float ssum = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    ids[j] = 0;
    psel[j] = 0.f;
    if (j < k) {
      int best = -1;
      float bv = 0.f;
#pragma unroll
      for (int i = 0; i < MAXE; ++i) {
        if (i < E && !((sel >> i) & 1ull) && (best < 0 || l[i] > bv)) {
          best = i;
          bv = l[i];
        }
      }
      sel |= 1ull << best;
      ids[j] = best;
      float pb = 0.f;
#pragma unroll
      for (int i = 0; i < MAXE; ++i)
        if (i == best) pb = p[i];
      psel[j] = pb;
      ssum += pb;
    }
  }
  const float denom = ssum + 1e-9f;
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) wsel[j] = psel[j] / denom;
}

template <int MAXE>
LR_DEVICE void warp_prob_sums(const float (&p)[MAXE], int E, float* s_pw) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < MAXE; ++i) {
    if (i < E) {
      float v = p[i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) s_pw[warp * E + i] = v;
    }
  }
}

template <int MAXE>
__global__ void __launch_bounds__(kRouteThreads)
    topk_route_kernel(const float* __restrict__ logits, int T, int E, int k, int C, float lbw,
                      int32_t* __restrict__ expert_ids, float* __restrict__ gate_w,
                      int32_t* __restrict__ token_idx, int32_t* __restrict__ slot_rank,
                      int32_t* __restrict__ offsets, int32_t* __restrict__ kept_counts,
                      float* __restrict__ aux_loss, double* __restrict__ prob_sums, RouteWs ws,
                      int num_blocks) {
  __shared__ int32_t s_ids[kRouteThreads * kMaxTopK];
  __shared__ int32_t s_wcnt[kWarps * MAXE];
  __shared__ int32_t s_run[MAXE];
  __shared__ float s_pw[kWarps * MAXE];
  __shared__ double s_P[MAXE];
  __shared__ int32_t s_tot[MAXE];
  __shared__ int s_last;

  const int tid = threadIdx.x;
  const int t = blockIdx.x * kRouteThreads + tid;
  const bool valid = t < T;
  const int ntok = min(kRouteThreads, T - int(blockIdx.x) * kRouteThreads);
  const int nslots = ntok * k;
  for (int i = tid; i < E; i += kRouteThreads) s_run[i] = 0;

  float p[MAXE];
  {
    float l[MAXE];
    const float* row = logits + size_t(valid ? t : 0) * E;
#pragma unroll
    for (int i = 0; i < MAXE; ++i) l[i] = (i < E && valid) ? __ldg(row + i) : 0.f;
    int ids[kMaxTopK];
    float wsel[kMaxTopK];
    topk_softmax<MAXE>(l, E, k, p, ids, wsel);
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) {
      if (j < k) {
        s_ids[tid * k + j] = ids[j];
        if (valid) {
          const size_t s = size_t(t) * k + j;
          expert_ids[s] = ids[j];
          gate_w[s] = wsel[j];
          if (token_idx) token_idx[s] = t;
        }
      }
    }
  }
  if (!valid) {
#pragma unroll
    for (int i = 0; i < MAXE; ++i) p[i] = 0.f;
  }
  // per-warp probability sums (aux loss)
  const bool want_p = aux_loss != nullptr || prob_sums != nullptr;
  if (want_p) warp_prob_sums<MAXE>(p, E, s_pw);
  __syncthreads();

  // slot ranks, chunk by chunk in slot order
  const size_t slot0 = size_t(blockIdx.x) * kRouteThreads * k;
  for (int c = 0; c < k; ++c) {
    const int ls = c * kRouteThreads + tid;
    const bool sv = ls < nslots;
    const int e = sv ? s_ids[ls] : -1;
    const int r = rank_chunk(e, sv, E, s_wcnt, s_run);
    if (sv) slot_rank[slot0 + ls] = r;
  }
  for (int i = tid; i < E; i += kRouteThreads) {
    ws.blk_counts[size_t(blockIdx.x) * E + i] = s_run[i];
    if (want_p) {
      double sum = 0.0;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) sum += double(s_pw[w * E + i]);
      ws.blk_psum[size_t(blockIdx.x) * E + i] = sum;
    }
  }
  if (!arrive_last(ws.ticket, num_blocks, &s_last)) return;
  route_tail(ws, num_blocks, E, C, T * k, T, k, lbw, offsets, kept_counts, aux_loss, prob_sums,
             s_tot, s_P);
}

// ---------------------------------------------------------------------------
// given-ids route: slot ranks + histogram
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kRouteThreads)
    slot_route_kernel(const int32_t* __restrict__ expert_ids, int S, int E, int C,
                      int32_t* __restrict__ slot_rank, int32_t* __restrict__ offsets,
                      int32_t* __restrict__ kept_counts, RouteWs ws, int num_blocks,
                      int32_t* err) {
  extern __shared__ int32_t dyn[];
  int32_t* s_wcnt = dyn;                 // kWarps * E
  int32_t* s_run = dyn + kWarps * E;     // E
  int32_t* s_tot = s_run + E;            // E
  double* s_P = reinterpret_cast<double*>(dyn + ((kWarps * E + 2 * E + 3) & ~3));  // E, 16B-aligned
  __shared__ int s_last;
  const int tid = threadIdx.x;
  for (int i = tid; i < E; i += kRouteThreads) s_run[i] = 0;
  __syncthreads();
  const size_t base = size_t(blockIdx.x) * kSlotBlock;
  for (int c = 0; c < kSlotBlock / kRouteThreads; ++c) {
    const size_t s = base + size_t(c) * kRouteThreads + tid;
    int e = -1;
    bool v = s < size_t(S);
    if (v) {
      e = __ldg(expert_ids + s);
      if (e < 0 || e >= E) {
        report(err, LR_DEVERR_BAD_EXPERT);
        v = false;
        e = -1;
      }
    }
    const int r = rank_chunk(e, v, E, s_wcnt, s_run);
    if (s < size_t(S)) slot_rank[s] = r;  // -1 marks an invalid slot
  }
  for (int i = tid; i < E; i += kRouteThreads) ws.blk_counts[size_t(blockIdx.x) * E + i] = s_run[i];
  if (!arrive_last(ws.ticket, num_blocks, &s_last)) return;
  route_tail(ws, num_blocks, E, C, S, 1, 1, 0.f, offsets, kept_counts, nullptr, nullptr, s_tot,
             s_P);
}

// ---------------------------------------------------------------------------
// permute
// ---------------------------------------------------------------------------
constexpr int kCopyUnroll = 8;

// One warp copies 16-byte chunks [c_beg, c_end) of a token row to the rows of
// its k slots.  Lane j < k holds slot j's destination row (`my_dst`, -1 for
// none) and whether it is kept; a dropped slot's row is zero-filled iff `fill`.
LR_DEVICE void copy_token_rows(const uint4* __restrict__ src, int c_beg, int c_end, int d8, int k,
                               int my_dst, int my_kept, int fill, uint4* __restrict__ permuted) {
  const int lane = threadIdx.x & 31;
  int dst[kMaxTopK];
  unsigned keptm = 0;
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    dst[j] = __shfl_sync(0xffffffffu, my_dst, j);
    keptm |= unsigned(__shfl_sync(0xffffffffu, my_kept, j) != 0) << j;
  }
  const uint4 zero = make_uint4(0, 0, 0, 0);
  for (int c0 = c_beg; c0 < c_end; c0 += 32 * kCopyUnroll) {
    uint4 v[kCopyUnroll];
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < c_end) v[u] = ld_stream(src + c);
    }
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) {
      if (j < k && dst[j] >= 0 && (((keptm >> j) & 1u) || fill)) {
        uint4* o = permuted + size_t(dst[j]) * d8;
        const bool kj = (keptm >> j) & 1u;
#pragma unroll
        for (int u = 0; u < kCopyUnroll; ++u) {
          const int c = c0 + u * 32 + lane;
          if (c < c_end) o[c] = kj ? v[u] : zero;
        }
      }
    }
  }
}

// gated routing: one warp per token, the row is read once and written k times.
// A slot's rank inside this shard's expert segment is blk_base + block rank;
// its expert-wide rank adds rank_base[e] (the slots of lower shards, or 0).
// It is kept iff the expert-wide rank < C and lands at row_offsets[e] + rank.
// With `compact`, dropped slots get no row (row_offsets then counts kept rows only).
__global__ void __launch_bounds__(256)
    permute_tokens_kernel(const uint4* __restrict__ x, int T, int d8, int k, int E, int C,
                          int fill, const int32_t* __restrict__ expert_ids,
                          const float* __restrict__ gate_w, const int32_t* __restrict__ offsets,
                          const int32_t* __restrict__ rank_base, int compact,
                          const int32_t* __restrict__ blk_base, int slots_per_blk,
                          int32_t* __restrict__ slot_pos, uint4* __restrict__ permuted,
                          float* __restrict__ routing_w, int32_t* __restrict__ src_idx) {
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  int my_dst = -1, my_kept = 0;
  if (lane < k) {
    const size_t s = size_t(t) * k + lane;
    const int e = expert_ids[s];
    const int r = slot_pos[s];
    const int rank = __ldg(blk_base + size_t(s / slots_per_blk) * E + e) + r;
    my_kept = (rank_base ? __ldg(rank_base + e) : 0) + rank < C;
    if (my_kept || !compact) {
      my_dst = __ldg(offsets + e) + rank;
      routing_w[my_dst] = my_kept ? gate_w[s] : 0.f;
      src_idx[my_dst] = t;
    }
    slot_pos[s] = my_kept ? my_dst : -1;
  }
  if (permuted == nullptr) return;
  copy_token_rows(x + size_t(t) * d8, 0, d8, d8, k, my_dst, my_kept, fill, permuted);
}

// given slots: one warp per slot, row x[token_idx[s]] -> permuted[dst].
__global__ void __launch_bounds__(256)
    permute_slots_kernel(const uint4* __restrict__ x, int T, int d8, int S, int E, int C,
                         int fill, const int32_t* __restrict__ expert_ids,
                         const float* __restrict__ gate_w, const int32_t* __restrict__ token_idx,
                         const int32_t* __restrict__ offsets, const int32_t* __restrict__ blk_base,
                         int32_t* __restrict__ slot_pos, uint4* __restrict__ permuted,
                         float* __restrict__ routing_w, int32_t* __restrict__ src_idx,
                         int32_t* err) {
  const int s = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (s >= S) return;
  const int lane = threadIdx.x & 31;
  int dst = -1, kept = 0, tok = 0;
  if (lane == 0) {
    const int r = slot_pos[s];
    if (r >= 0) {
      const int e = expert_ids[s];
      const int rank = __ldg(blk_base + size_t(s / kSlotBlock) * E + e) + r;
      dst = __ldg(offsets + e) + rank;
      kept = rank < C;
      tok = token_idx[s];
      if (tok < 0 || tok >= T) {
        report(err, LR_DEVERR_BAD_TOKEN);
        kept = 0;
        tok = 0;
      }
      slot_pos[s] = kept ? dst : -1;
      routing_w[dst] = kept ? gate_w[s] : 0.f;
      src_idx[dst] = tok;
    } else {
      slot_pos[s] = -1;
    }
  }
  dst = __shfl_sync(0xffffffffu, dst, 0);
  kept = __shfl_sync(0xffffffffu, kept, 0);
  tok = __shfl_sync(0xffffffffu, tok, 0);
  if (permuted == nullptr || dst < 0 || (!kept && !fill)) return;
  const uint4* srcp = x + size_t(tok) * d8;
  uint4* o = permuted + size_t(dst) * d8;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  for (int c0 = 0; c0 < d8; c0 += 32 * kCopyUnroll) {
    uint4 v[kCopyUnroll];
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < d8) v[u] = kept ? ld_stream(srcp + c) : zero;
    }
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < d8) o[c] = v[u];
    }
  }
}

// ---------------------------------------------------------------------------
// small batches (decode): gate projection + top-k + ranks + rows in one launch
// ---------------------------------------------------------------------------
// For T <= 256 tokens a single block can rank every slot, so the route needs
// no per-block bases.  The gate projection is spread over blocks by
// (d-chunk c of kGateWarps, 16-token tile), warp w taking experts
// [8w, 8w + 8): chunk c covers the k range of warp c of gate_logits_kernel
// with the same mma.sync sequence per 8-expert group, and the last block to
// finish sums the chunk partials in chunk order and adds the bias as that
// kernel does, so the logits are bit-identical to the two-kernel path.
// That block then runs top-k, ranks, CSR offsets, capacity and the aux loss for
// all tokens and writes each slot's row; permute_rows_kernel copies the rows.
constexpr int kSmallTokens = kRouteThreads;  // token limit of the one-block route
constexpr int kSgTok = 16;                   // tokens per gate block (one mma tile)
constexpr int kSgPiece = 512;                // k per shared-memory piece
constexpr int kSgLd = kSgPiece + 8;          // padded row in halves: rows 4 banks apart

struct SmallRouteWs {
  int32_t* ticket;
  float* part;        // [kGateWarps][T][E] partial logits
  int32_t* slot_row;  // [T*k] row of each slot (dropped slots included)
};

static size_t small_route_ws_bytes(int T, int k, int E) {
  return 256 + align256(size_t(kGateWarps) * T * E * sizeof(float)) +
         align256(size_t(T) * k * sizeof(int32_t));
}

static SmallRouteWs carve_small_route_ws(void* ws, int T, int E) {
  char* p = static_cast<char*>(ws);
  SmallRouteWs r;
  r.ticket = reinterpret_cast<int32_t*>(p);
  p += 256;
  r.part = reinterpret_cast<float*>(p);
  p += align256(size_t(kGateWarps) * T * E * sizeof(float));
  r.slot_row = reinterpret_cast<int32_t*>(p);
  return r;
}

static size_t small_gate_smem_bytes(int E) {
  return size_t(kSgTok + ((E + 7) & ~7)) * kSgLd * sizeof(__half);
}

// 16-byte global -> shared copy; with pred false the destination is zero-filled
// and nothing is read.
LR_DEVICE void cp_async16(uint32_t saddr, const void* gptr, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr), "l"(gptr),
               "r"(pred ? 16 : 0)
               : "memory");
}
LR_DEVICE void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
LR_DEVICE uint32_t lds_u32(const __half* p) { return *reinterpret_cast<const uint32_t*>(p); }

template <int MAXE>
__global__ void __launch_bounds__(kRouteThreads)
    gate_route_small_kernel(const __half* __restrict__ h, const __half* __restrict__ wg,
                            const float* __restrict__ bias, int T, int d, int E, int k, int C,
                            float lbw, float* __restrict__ logits,
                            int32_t* __restrict__ expert_ids, float* __restrict__ gate_w,
                            int32_t* __restrict__ token_idx, int32_t* __restrict__ offsets,
                            int32_t* __restrict__ kept_counts, float* __restrict__ aux_loss,
                            float* __restrict__ routing_w, int32_t* __restrict__ src_idx,
                            int32_t* __restrict__ slot_pos, SmallRouteWs ws, int num_blocks) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) __half s_gate[];  // [kSgTok][kSgLd] tokens, [Epad][kSgLd] gate
  __shared__ int32_t s_ids[kRouteThreads * kMaxTopK];
  __shared__ int32_t s_rank[kRouteThreads * kMaxTopK];
  __shared__ int32_t s_wcnt[kWarps * MAXE];
  __shared__ int32_t s_run[MAXE];
  __shared__ int32_t s_off[MAXE];
  __shared__ float s_pw[kWarps * MAXE];
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, tq = lane & 3;

  // ---- gate partials of d-chunk `chunk` for tokens [t0, t0 + 16)
  {
    const int chunk = blockIdx.x % kGateWarps;
    const int t0 = (blockIdx.x / kGateWarps) * kSgTok;
    const int kc = ((d / 16 + kGateWarps - 1) / kGateWarps) * 16;
    const int kbeg = chunk * kc, kend = min(d, kbeg + kc);
    const int epad = (E + 7) & ~7;
    __half* s_h = s_gate;
    __half* s_w = s_gate + kSgTok * kSgLd;
    const int e0 = warp * 8;  // this warp's 8 experts
    const bool active = e0 < E;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int p0 = kbeg; p0 < kend; p0 += kSgPiece) {
      const int L = min(kSgPiece, kend - p0);  // a multiple of 16
      const int cpr = L / 8;                    // 16-byte chunks per row
      __syncthreads();                          // the previous piece is consumed
      for (int i = tid; i < kSgTok * cpr; i += kRouteThreads) {
        const int r = i / cpr, c = i - r * cpr;
        const bool ok = t0 + r < T;
        cp_async16(smem_u32(s_h + r * kSgLd + c * 8),
                   h + size_t(ok ? t0 + r : 0) * d + p0 + c * 8, ok);
      }
      for (int i = tid; i < epad * cpr; i += kRouteThreads) {
        const int r = i / cpr, c = i - r * cpr;
        const bool ok = r < E;
        cp_async16(smem_u32(s_w + r * kSgLd + c * 8), wg + size_t(ok ? r : 0) * d + p0 + c * 8,
                   ok);
      }
      cp_async_wait_all();
      __syncthreads();
      if (active) {
        const __half* a0 = s_h + g * kSgLd + 2 * tq;
        const __half* a1 = a0 + 8 * kSgLd;
        const __half* b = s_w + (e0 + g) * kSgLd + 2 * tq;
#pragma unroll 4
        for (int kk = 0; kk < L; kk += 16) {
          uint32_t a[4];
          a[0] = lds_u32(a0 + kk);
          a[1] = lds_u32(a1 + kk);
          a[2] = lds_u32(a0 + kk + 8);
          a[3] = lds_u32(a1 + kk + 8);
          mma_16816(acc, a, lds_u32(b + kk), lds_u32(b + kk + 8));
        }
      }
    }
    if (active) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = t0 + ((i < 2) ? g : g + 8);
        const int col = e0 + 2 * tq + (i & 1);
        if (row < T && col < E) ws.part[(size_t(chunk) * T + row) * E + col] = acc[i];
      }
    }
  }
  if (!arrive_last(ws.ticket, num_blocks, &s_last)) return;

  // ---- last block: logits, top-k, ranks, offsets, rows (thread = token)
  for (int i = tid; i < E; i += kRouteThreads) s_run[i] = 0;
  const int t = tid;
  const bool valid = t < T;
  float p[MAXE];
  int ids[kMaxTopK];
  float wsel[kMaxTopK];
  {
    float l[MAXE];
#pragma unroll
    for (int i = 0; i < MAXE; ++i) {
      float v = 0.f;
      if (i < E && valid) {
#pragma unroll
        for (int c = 0; c < kGateWarps; ++c) v += __ldcg(ws.part + (size_t(c) * T + t) * E + i);
        if (bias) v += __ldg(bias + i);
        if (logits) logits[size_t(t) * E + i] = v;
      }
      l[i] = v;
    }
    topk_softmax<MAXE>(l, E, k, p, ids, wsel);
  }
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    if (j < k) {
      s_ids[tid * k + j] = ids[j];
      if (valid) {
        const size_t s = size_t(t) * k + j;
        expert_ids[s] = ids[j];
        gate_w[s] = wsel[j];
        if (token_idx) token_idx[s] = t;
      }
    }
  }
  if (!valid) {
#pragma unroll
    for (int i = 0; i < MAXE; ++i) p[i] = 0.f;
  }
  if (aux_loss) warp_prob_sums<MAXE>(p, E, s_pw);
  __syncthreads();
  const int nslots = T * k;
  for (int c = 0; c < k; ++c) {
    const int ls = c * kRouteThreads + tid;
    const bool sv = ls < nslots;
    const int r = rank_chunk(sv ? s_ids[ls] : -1, sv, E, s_wcnt, s_run);
    if (sv) s_rank[ls] = r;
  }
  // s_run[e] now counts expert e's slots (uncapped)
  if (tid == 0) {
    int run = 0;
    double aux = 0.0;
    offsets[0] = 0;
    for (int e = 0; e < E; ++e) {
      s_off[e] = run;
      run += s_run[e];
      offsets[e + 1] = run;
      if (kept_counts) kept_counts[e] = min(s_run[e], C);
      if (aux_loss) {
        double P = 0.0;
        for (int w = 0; w < kWarps; ++w) P += double(s_pw[w * E + e]);
        aux += (double(s_run[e]) / double(nslots)) * (P / double(T));
      }
    }
    if (aux_loss) aux_loss[0] = static_cast<float>(double(lbw) * double(E) * aux);
    *ws.ticket = 0;
  }
  __syncthreads();
  if (valid) {
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) {
      if (j < k) {
        const int s = t * k + j;
        const int r = s_rank[tid * k + j];
        const bool kept = r < C;
        const int dst = s_off[ids[j]] + r;
        routing_w[dst] = kept ? wsel[j] : 0.f;
        src_idx[dst] = t;
        slot_pos[s] = kept ? dst : -1;
        ws.slot_row[s] = dst;
      }
    }
  }
}

// Row copy after gate_route_small_kernel: one warp per (token, 1/parts of the row).
__global__ void __launch_bounds__(256)
    permute_rows_kernel(const uint4* __restrict__ x, int T, int d8, int k, int parts, int fill,
                        const int32_t* __restrict__ slot_pos,
                        const int32_t* __restrict__ slot_row, uint4* __restrict__ permuted) {
  pdl_wait();
  pdl_trigger();
  const int gw = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int t = gw / parts, part = gw % parts;
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  int my_dst = -1, my_kept = 0;
  if (lane < k) {
    const size_t s = size_t(t) * k + lane;
    my_dst = __ldg(slot_row + s);
    my_kept = __ldg(slot_pos + s) >= 0;
  }
  const int seg = (d8 + parts - 1) / parts;
  const int c_beg = part * seg, c_end = min(d8, c_beg + seg);
  copy_token_rows(x + size_t(t) * d8, c_beg, c_end, d8, k, my_dst, my_kept, fill, permuted);
}

// ---------------------------------------------------------------------------
// combine: one warp per (token, 1/parts of the row), fp32 accumulation in
// slot order (the split only spreads small batches over more warps)
// ---------------------------------------------------------------------------
constexpr int kCombUnroll = 4;

// Row parts per token: enough warps in flight for small batches, each part
// at least 64 16-byte chunks.
static int row_parts(long T, int d8) {
  int parts = 1;
  while (parts < 8 && T * parts < 2048 && d8 / (parts * 2) >= 64) parts *= 2;
  return parts;
}

__global__ void __launch_bounds__(256)
    combine_kernel(const uint4* __restrict__ y, const float* __restrict__ gate_w,
                   const int32_t* __restrict__ slot_pos, int T, int k, int d8, int parts,
                   uint4* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int gw = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int t = gw / parts, part = gw % parts;
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  const int seg = (d8 + parts - 1) / parts;
  const int c_beg = part * seg, c_end = min(d8, c_beg + seg);
  int my_pos = -1;
  float my_w = 0.f;
  if (lane < k) {
    my_pos = __ldg(slot_pos + size_t(t) * k + lane);
    my_w = __ldg(gate_w + size_t(t) * k + lane);
  }
  int pos[kMaxTopK];
  float w[kMaxTopK];
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    pos[j] = __shfl_sync(0xffffffffu, my_pos, j);
    w[j] = __shfl_sync(0xffffffffu, my_w, j);
  }
  for (int c0 = c_beg; c0 < c_end; c0 += 32 * kCombUnroll) {
    float acc[kCombUnroll][8];
#pragma unroll
    for (int u = 0; u < kCombUnroll; ++u)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[u][i] = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) {
      if (j < k && pos[j] >= 0) {
        const uint4* row = y + size_t(pos[j]) * d8;
        uint4 v[kCombUnroll];
#pragma unroll
        for (int u = 0; u < kCombUnroll; ++u) {
          const int c = c0 + u * 32 + lane;
          if (c < c_end) v[u] = ld_stream(row + c);
        }
#pragma unroll
        for (int u = 0; u < kCombUnroll; ++u) {
          const int c = c0 + u * 32 + lane;
          if (c < c_end) acc_half8(acc[u], v[u], w[j]);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kCombUnroll; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < c_end) out[size_t(t) * d8 + c] = pack_half8(acc[u]);
    }
  }
}

// ---------------------------------------------------------------------------
// general gather (rows -> tokens), deterministic
// ---------------------------------------------------------------------------
__global__ void gather_count_kernel(const float* __restrict__ rw, const int32_t* __restrict__ src,
                                    int R, int T, int32_t* __restrict__ cnt, int32_t* err) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= R) return;
  if (rw[r] == 0.f) return;
  const int t = src[r];
  if (t < 0 || t >= T) {
    report(err, LR_DEVERR_BAD_TOKEN);
    return;
  }
  atomicAdd(cnt + t, 1);
}

// single-block exclusive scan of cnt[0..n) into off[0..n]
__global__ void __launch_bounds__(1024) scan_kernel(const int32_t* __restrict__ cnt, int n,
                                                    int32_t* __restrict__ off) {
  __shared__ int32_t s_warp[32];
  __shared__ int32_t s_carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_carry = 0;
  __syncthreads();
  for (int base = 0; base < n; base += 1024) {
    const int i = base + tid;
    const int v = i < n ? cnt[i] : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += x;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int wv = s_warp[lane];
      int wi = wv;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int x = __shfl_up_sync(0xffffffffu, wi, o);
        if (lane >= o) wi += x;
      }
      s_warp[lane] = wi - wv;
    }
    __syncthreads();
    const int carry = s_carry;
    if (i < n) off[i] = carry + s_warp[warp] + incl - v;
    __syncthreads();
    if (tid == 1023) s_carry = carry + s_warp[warp] + incl;
    __syncthreads();
  }
  if (tid == 0) off[n] = s_carry;
}

__global__ void gather_fill_kernel(const float* __restrict__ rw, const int32_t* __restrict__ src,
                                   int R, int T, const int32_t* __restrict__ off,
                                   int32_t* __restrict__ fillc, int32_t* __restrict__ list) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= R) return;
  if (rw[r] == 0.f) return;
  const int t = src[r];
  if (t < 0 || t >= T) return;
  list[off[t] + atomicAdd(fillc + t, 1)] = r;
}

// one warp per token: order the token's rows ascending (selection), then
// accumulate w * y in that order in fp32.
__global__ void __launch_bounds__(256)
    gather_combine_kernel(const uint4* __restrict__ y, const float* __restrict__ rw,
                          const int32_t* __restrict__ off, const int32_t* __restrict__ list,
                          int32_t* __restrict__ sorted, int T, int d8, uint4* __restrict__ out) {
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  const int b = off[t], n = off[t + 1] - b;
  int prev = -1;
  for (int q = 0; q < n; ++q) {
    int best = 0x7fffffff;
    for (int i = lane; i < n; i += 32) {
      const int r = list[b + i];
      if (r > prev && r < best) best = r;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = min(best, __shfl_xor_sync(0xffffffffu, best, o));
    if (lane == 0) sorted[b + q] = best;
    prev = best;
  }
  __syncwarp();
  for (int c0 = 0; c0 < d8; c0 += 32 * kCombUnroll) {
    float acc[kCombUnroll][8];
#pragma unroll
    for (int u = 0; u < kCombUnroll; ++u)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[u][i] = 0.f;
    for (int q = 0; q < n; ++q) {
      const int r = sorted[b + q];
      const float w = rw[r];
      const uint4* row = y + size_t(r) * d8;
#pragma unroll
      for (int u = 0; u < kCombUnroll; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < d8) acc_half8(acc[u], ld_stream(row + c), w);
      }
    }
#pragma unroll
    for (int u = 0; u < kCombUnroll; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < d8) out[size_t(t) * d8 + c] = pack_half8(acc[u]);
    }
  }
}

}  // namespace lr

// ===========================================================================
// C ABI
// ===========================================================================
using namespace lr;

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" int lr_gate_logits(const void* h, const void* wg, const float* bias, int T, int d, int E,
                              float* logits, lr_stream_t stream) {
  if (T < 0 || d <= 0 || d % 16 != 0 || E < 1 || E > 256) return LR_ERR_INVALID_ARGUMENT;
  if (T == 0) return LR_OK;
  if (!h || !wg || !logits) return LR_ERR_INVALID_ARGUMENT;
  const int n_eg = (E + 31) / 32;
  const long blocks = long((T + 15) / 16) * n_eg;
  gate_logits_kernel<<<unsigned(blocks), kGateWarps * 32, 0, stream>>>(static_cast<const __half*>(h),
                                                 static_cast<const __half*>(wg), bias, T, d, E,
                                                 n_eg, logits);
  LR_LAUNCH_CHECK();
  return LR_OK;
}

extern "C" size_t lr_route_workspace_bytes(int num_tokens, int top_k, int num_experts) {
  const int B = (num_tokens + kRouteThreads - 1) / kRouteThreads;
  (void)top_k;
  return route_ws_bytes_for(B < 1 ? 1 : B, num_experts, true);
}

extern "C" int lr_topk_route(const float* logits, int T, int E, int k, int capacity,
                             float load_balance_weight, int32_t* expert_ids, float* gate_weights,
                             int32_t* token_indices, int32_t* offsets, int32_t* kept_counts,
                             float* aux_loss, double* prob_sums, int32_t* slot_pos,
                             void* workspace, size_t workspace_bytes, int32_t* err,
                             lr_stream_t stream) {
  (void)err;
  if (T <= 0 || E < 1 || E > 64 || k < 1 || k > kMaxTopK || k > E || capacity < 1)
    return LR_ERR_INVALID_ARGUMENT;
  if (!logits || !expert_ids || !gate_weights || !offsets || !slot_pos)
    return LR_ERR_INVALID_ARGUMENT;
  const int B = (T + kRouteThreads - 1) / kRouteThreads;
  if (!workspace || workspace_bytes < route_ws_bytes_for(B, E, true)) return LR_ERR_WORKSPACE;
  RouteWs ws = carve_route_ws(workspace, B, E, true);
  LR_CUDA_TRY(cudaMemsetAsync(ws.ticket, 0, sizeof(int32_t), stream));
#define LR_ROUTE_CASE(ME)                                                                      \
  topk_route_kernel<ME><<<B, kRouteThreads, 0, stream>>>(                                      \
      logits, T, E, k, capacity, load_balance_weight, expert_ids, gate_weights, token_indices, \
      slot_pos, offsets, kept_counts, aux_loss, prob_sums, ws, B)
  if (E <= 8)
    LR_ROUTE_CASE(8);
  else if (E <= 16)
    LR_ROUTE_CASE(16);
  else if (E <= 32)
    LR_ROUTE_CASE(32);
  else
    LR_ROUTE_CASE(64);
#undef LR_ROUTE_CASE
  LR_LAUNCH_CHECK();
  return LR_OK;
}

extern "C" int lr_permute_tokens(const void* x, int T, int d, int E, int k, int capacity,
                                 const int32_t* expert_ids, const float* gate_weights,
                                 const int32_t* row_offsets, const int32_t* rank_base,
                                 int compact, int fill_dropped, int32_t* slot_pos, void* permuted,
                                 float* routing_w, int32_t* source_idx, const void* workspace,
                                 size_t workspace_bytes, lr_stream_t stream) {
  if (T <= 0 || E < 1 || E > 64 || k < 1 || k > kMaxTopK || k > E || capacity < 1)
    return LR_ERR_INVALID_ARGUMENT;
  if (!expert_ids || !gate_weights || !row_offsets || !slot_pos || !routing_w || !source_idx)
    return LR_ERR_INVALID_ARGUMENT;
  if (permuted && (!x || d <= 0 || d % 8 != 0 || !aligned16(x) || !aligned16(permuted)))
    return LR_ERR_INVALID_ARGUMENT;
  const int B = (T + kRouteThreads - 1) / kRouteThreads;
  if (!workspace || workspace_bytes < route_ws_bytes_for(B, E, true)) return LR_ERR_WORKSPACE;
  RouteWs ws = carve_route_ws(const_cast<void*>(workspace), B, E, true);
  permute_tokens_kernel<<<(T + 7) / 8, 256, 0, stream>>>(
      static_cast<const uint4*>(x), T, d / 8, k, E, capacity, fill_dropped, expert_ids,
      gate_weights, row_offsets, rank_base, compact, ws.blk_base, kRouteThreads * k, slot_pos,
      static_cast<uint4*>(permuted), routing_w, source_idx);
  LR_LAUNCH_CHECK();
  return LR_OK;
}

extern "C" int lr_topk_gating_dispatch(const void* x, const float* logits, int T, int d, int E,
                                       int k, int capacity, float load_balance_weight,
                                       int fill_dropped, int32_t* expert_ids, float* gate_weights,
                                       int32_t* token_indices, int32_t* offsets,
                                       int32_t* kept_counts, float* aux_loss, void* permuted,
                                       float* routing_w, int32_t* source_idx, int32_t* slot_pos,
                                       void* workspace, size_t workspace_bytes, int32_t* err,
                                       lr_stream_t stream) {
  if (!routing_w || !source_idx) return LR_ERR_INVALID_ARGUMENT;
  if (permuted && (!x || d <= 0 || d % 8 != 0 || !aligned16(x) || !aligned16(permuted)))
    return LR_ERR_INVALID_ARGUMENT;
  int rc = lr_topk_route(logits, T, E, k, capacity, load_balance_weight, expert_ids, gate_weights,
                         token_indices, offsets, kept_counts, aux_loss, nullptr, slot_pos,
                         workspace, workspace_bytes, err, stream);
  if (rc != LR_OK) return rc;
  return lr_permute_tokens(x, T, d, E, k, capacity, expert_ids, gate_weights, offsets, nullptr, 0,
                           fill_dropped, slot_pos, permuted, routing_w, source_idx, workspace,
                           workspace_bytes, stream);
}

extern "C" size_t lr_gate_dispatch_workspace_bytes(int num_tokens, int top_k, int num_experts) {
  const size_t big = lr_route_workspace_bytes(num_tokens, top_k, num_experts);
  if (num_tokens < 1 || num_tokens > kSmallTokens || top_k < 1 || num_experts < 1) return big;
  const size_t small = small_route_ws_bytes(num_tokens, top_k, num_experts);
  return small > big ? small : big;
}

template <int MAXE>
static int launch_gate_route_small(const void* x, const void* wg, const float* bias, int T, int d,
                                   int E, int k, int capacity, float lbw, float* logits,
                                   int32_t* expert_ids, float* gate_weights,
                                   int32_t* token_indices, int32_t* offsets,
                                   int32_t* kept_counts, float* aux_loss, float* routing_w,
                                   int32_t* source_idx, int32_t* slot_pos, SmallRouteWs ws,
                                   cudaStream_t stream) {
  auto kern = gate_route_small_kernel<MAXE>;
  static unsigned long long configured = 0;
  if (const int rc = set_dyn_smem_once(kern, int(small_gate_smem_bytes(64)), configured)) return rc;
  const int blocks = kGateWarps * ((T + kSgTok - 1) / kSgTok);
  if (const int rc = launch_pdl(kern, dim3(blocks), dim3(kRouteThreads), small_gate_smem_bytes(E),
                               stream, static_cast<const __half*>(x),
                               static_cast<const __half*>(wg), bias, T, d, E, k, capacity, lbw,
                               logits, expert_ids, gate_weights, token_indices, offsets,
                               kept_counts, aux_loss, routing_w, source_idx, slot_pos, ws, blocks))
    return rc;
  return LR_OK;
}

extern "C" int lr_gate_topk_gating_dispatch(
    const void* x, const void* gate_weight, const float* bias, int T, int d, int E, int k,
    int capacity, float load_balance_weight, int fill_dropped, float* logits,
    int32_t* expert_ids, float* gate_weights, int32_t* token_indices, int32_t* offsets,
    int32_t* kept_counts, float* aux_loss, void* permuted, float* routing_w, int32_t* source_idx,
    int32_t* slot_pos, void* workspace, size_t workspace_bytes, int32_t* err,
    lr_stream_t stream) {
  if (T <= 0 || d <= 0 || d % 16 != 0 || E < 1 || E > 64 || k < 1 || k > kMaxTopK || k > E ||
      capacity < 1)
    return LR_ERR_INVALID_ARGUMENT;
  if (!x || !gate_weight || !logits || !expert_ids || !gate_weights || !offsets || !routing_w ||
      !source_idx || !slot_pos)
    return LR_ERR_INVALID_ARGUMENT;
  if (!aligned16(x) || !aligned16(gate_weight) || (permuted && !aligned16(permuted)))
    return LR_ERR_INVALID_ARGUMENT;
  if (T > kSmallTokens) {
    const int rc = lr_gate_logits(x, gate_weight, bias, T, d, E, logits, stream);
    if (rc != LR_OK) return rc;
    return lr_topk_gating_dispatch(x, logits, T, d, E, k, capacity, load_balance_weight,
                                   fill_dropped, expert_ids, gate_weights, token_indices, offsets,
                                   kept_counts, aux_loss, permuted, routing_w, source_idx,
                                   slot_pos, workspace, workspace_bytes, err, stream);
  }
  if (!workspace || workspace_bytes < small_route_ws_bytes(T, k, E)) return LR_ERR_WORKSPACE;
  SmallRouteWs ws = carve_small_route_ws(workspace, T, E);
  LR_CUDA_TRY(cudaMemsetAsync(ws.ticket, 0, sizeof(int32_t), stream));
  int rc;
#define LR_SMALL_CASE(ME)                                                                       \
  rc = launch_gate_route_small<ME>(x, gate_weight, bias, T, d, E, k, capacity,                  \
                                   load_balance_weight, logits, expert_ids, gate_weights,       \
                                   token_indices, offsets, kept_counts, aux_loss, routing_w,    \
                                   source_idx, slot_pos, ws, stream)
  if (E <= 8)
    LR_SMALL_CASE(8);
  else if (E <= 16)
    LR_SMALL_CASE(16);
  else if (E <= 32)
    LR_SMALL_CASE(32);
  else
    LR_SMALL_CASE(64);
#undef LR_SMALL_CASE
  if (rc != LR_OK || permuted == nullptr) return rc;
  const int parts = row_parts(T, d / 8);
  if (const int rc = launch_pdl(permute_rows_kernel, dim3(unsigned((long(T) * parts + 7) / 8)),
                               dim3(256), 0, stream, static_cast<const uint4*>(x), T, d / 8, k,
                               parts, fill_dropped, slot_pos, ws.slot_row,
                               static_cast<uint4*>(permuted)))
    return rc;
  return LR_OK;
}

extern "C" size_t lr_dispatch_workspace_bytes(int num_slots, int num_experts) {
  const int B = (num_slots + kSlotBlock - 1) / kSlotBlock;
  return route_ws_bytes_for(B < 1 ? 1 : B, num_experts, false);
}

extern "C" int lr_expert_routing_forward(const void* tokens, const int32_t* expert_ids,
                                         const float* gate_weights, const int32_t* token_indices,
                                         int T, int d, int S, int E, int capacity,
                                         int fill_dropped, void* permuted, int32_t* offsets,
                                         float* routing_w, int32_t* source_idx,
                                         int32_t* kept_counts, int32_t* slot_pos, void* workspace,
                                         size_t workspace_bytes, int32_t* err,
                                         lr_stream_t stream) {
  if (T < 0 || S < 0 || E < 1 || E > 1024 || capacity < 1) return LR_ERR_INVALID_ARGUMENT;
  if (!offsets) return LR_ERR_INVALID_ARGUMENT;
  if (S == 0) {
    LR_CUDA_TRY(cudaMemsetAsync(offsets, 0, sizeof(int32_t) * (E + 1), stream));
    if (kept_counts) LR_CUDA_TRY(cudaMemsetAsync(kept_counts, 0, sizeof(int32_t) * E, stream));
    return LR_OK;
  }
  if (!expert_ids || !gate_weights || !token_indices || !routing_w || !source_idx || !slot_pos)
    return LR_ERR_INVALID_ARGUMENT;
  if (permuted && (!tokens || d <= 0 || d % 8 != 0 || !aligned16(tokens) || !aligned16(permuted)))
    return LR_ERR_INVALID_ARGUMENT;
  const int B = (S + kSlotBlock - 1) / kSlotBlock;
  if (!workspace || workspace_bytes < route_ws_bytes_for(B, E, false)) return LR_ERR_WORKSPACE;
  RouteWs ws = carve_route_ws(workspace, B, E, false);
  LR_CUDA_TRY(cudaMemsetAsync(ws.ticket, 0, sizeof(int32_t), stream));
  const size_t smem = sizeof(int32_t) * ((kWarps * E + 2 * E + 3) & ~3) + sizeof(double) * E;
  if (smem > 48 * 1024)
    LR_CUDA_TRY(cudaFuncSetAttribute(slot_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     int(smem)));
  slot_route_kernel<<<B, kRouteThreads, smem, stream>>>(expert_ids, S, E, capacity, slot_pos,
                                                         offsets, kept_counts, ws, B, err);
  LR_LAUNCH_CHECK();
  permute_slots_kernel<<<(S + 7) / 8, 256, 0, stream>>>(
      static_cast<const uint4*>(tokens), T, d / 8, S, E, capacity, fill_dropped, expert_ids,
      gate_weights, token_indices, offsets, ws.blk_base, slot_pos, static_cast<uint4*>(permuted),
      routing_w, source_idx, err);
  LR_LAUNCH_CHECK();
  return LR_OK;
}

extern "C" int lr_combine(const void* y, const float* gate_weights, const int32_t* slot_pos, int T,
                          int k, int d, void* out, lr_stream_t stream) {
  if (T < 0 || k < 1 || k > kMaxTopK || d <= 0 || d % 8 != 0) return LR_ERR_INVALID_ARGUMENT;
  if (T == 0) return LR_OK;
  if (!y || !gate_weights || !slot_pos || !out || !aligned16(y) || !aligned16(out))
    return LR_ERR_INVALID_ARGUMENT;
  const int parts = row_parts(T, d / 8);
  if (const int rc = launch_pdl(combine_kernel, dim3(unsigned((long(T) * parts + 7) / 8)),
                               dim3(256), 0, stream, static_cast<const uint4*>(y), gate_weights,
                               slot_pos, T, k, d / 8, parts, static_cast<uint4*>(out)))
    return rc;
  return LR_OK;
}

extern "C" size_t lr_gather_workspace_bytes(int num_rows, int num_tokens) {
  size_t b = 0;
  b += align256(sizeof(int32_t) * size_t(num_tokens));       // cnt
  b += align256(sizeof(int32_t) * size_t(num_tokens));       // fill
  b += align256(sizeof(int32_t) * (size_t(num_tokens) + 1)); // off
  b += align256(sizeof(int32_t) * size_t(num_rows));         // list
  b += align256(sizeof(int32_t) * size_t(num_rows));         // sorted
  return b;
}

extern "C" int lr_expert_routing_gather(const void* y, const float* routing_w,
                                        const int32_t* source_idx, int R, int d, int T, void* out,
                                        void* workspace, size_t workspace_bytes, int32_t* err,
                                        lr_stream_t stream) {
  if (R < 0 || T < 0 || d <= 0 || d % 8 != 0) return LR_ERR_INVALID_ARGUMENT;
  if (T == 0) return LR_OK;
  if (!out || !aligned16(out)) return LR_ERR_INVALID_ARGUMENT;
  if (R > 0 && (!y || !routing_w || !source_idx || !aligned16(y))) return LR_ERR_INVALID_ARGUMENT;
  if (!workspace || workspace_bytes < lr_gather_workspace_bytes(R, T)) return LR_ERR_WORKSPACE;
  char* p = static_cast<char*>(workspace);
  int32_t* cnt = reinterpret_cast<int32_t*>(p);
  p += align256(sizeof(int32_t) * size_t(T));
  int32_t* fillc = reinterpret_cast<int32_t*>(p);
  p += align256(sizeof(int32_t) * size_t(T));
  int32_t* off = reinterpret_cast<int32_t*>(p);
  p += align256(sizeof(int32_t) * (size_t(T) + 1));
  int32_t* list = reinterpret_cast<int32_t*>(p);
  p += align256(sizeof(int32_t) * size_t(R));
  int32_t* sorted = reinterpret_cast<int32_t*>(p);
  LR_CUDA_TRY(cudaMemsetAsync(cnt, 0, 2 * align256(sizeof(int32_t) * size_t(T)), stream));
  if (R > 0) {
    gather_count_kernel<<<(R + 255) / 256, 256, 0, stream>>>(routing_w, source_idx, R, T, cnt, err);
    LR_LAUNCH_CHECK();
  }
  scan_kernel<<<1, 1024, 0, stream>>>(cnt, T, off);
  LR_LAUNCH_CHECK();
  if (R > 0) {
    gather_fill_kernel<<<(R + 255) / 256, 256, 0, stream>>>(routing_w, source_idx, R, T, off,
                                                            fillc, list);
    LR_LAUNCH_CHECK();
  }
  gather_combine_kernel<<<(T + 7) / 8, 256, 0, stream>>>(static_cast<const uint4*>(y), routing_w,
                                                         off, list, sorted, T, d / 8,
                                                         static_cast<uint4*>(out));
  LR_LAUNCH_CHECK();
  return LR_OK;
}

// ===========================================================================
// Allocation-free gating + dispatch
// ===========================================================================
// Some callers cannot allocate device memory: a serving host that owns every
// byte of device memory and hands this library pre-sized input and output
// buffers but no allocator, or a latency-critical loop that may not call
// cudaMalloc (it synchronises the whole device).  For them the route scratch
// lives in this file-scope device array instead of a caller workspace.  Every
// GPU that loads the library holds it until the process exits.
#include <cudaTypedefs.h>

#include <mutex>

static constexpr size_t kStaticRouteScratchBytes = size_t(1) << 20;  // 1 MiB
static __device__ __align__(256) unsigned char g_route_scratch[kStaticRouteScratchBytes];

static std::mutex g_route_scratch_mu;
// Device address per device ordinal, with the context it was found in.
struct RouteScratchAddr {
  CUcontext ctx;
  void* ptr;
};
static RouteScratchAddr g_route_scratch_dev[64];

static PFN_cuCtxGetCurrent_v4000 get_ctx_fn() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
  }
  return fn;
}

// Device address of g_route_scratch on the current device.  In host code the
// array's name is only a host-side stand-in, so the address is looked up with
// cudaGetSymbolAddress, with that device current, the first time the device's
// current context calls; a new context (after cudaDeviceReset, for one) looks
// it up again.  Ordinals of 64 and above are looked up on every call.
static int route_scratch_address(void** out) {
  int dev = 0;
  LR_CUDA_TRY(cudaGetDevice(&dev));
  auto ctx_fn = get_ctx_fn();
  // null until the runtime has made a context current on this thread
  auto current_ctx = [&]() -> CUcontext {
    CUcontext c = nullptr;
    if (!ctx_fn || ctx_fn(&c) != CUDA_SUCCESS) c = nullptr;
    return c;
  };
  CUcontext ctx = current_ctx();
  std::lock_guard<std::mutex> lock(g_route_scratch_mu);
  if (dev < 64 && ctx && g_route_scratch_dev[dev].ptr && g_route_scratch_dev[dev].ctx == ctx) {
    *out = g_route_scratch_dev[dev].ptr;
    return LR_OK;
  }
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_route_scratch);
  if (e != cudaSuccess || p == nullptr) return record_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
  if (dev < 64) g_route_scratch_dev[dev] = {current_ctx(), p};
  *out = p;
  return LR_OK;
}

extern "C" int lr_topk_gating_dispatch_noalloc(const void* x, const float* logits, int T, int d,
                                               int E, int k, int capacity,
                                               float load_balance_weight, int fill_dropped,
                                               int32_t* expert_ids, float* gate_weights,
                                               int32_t* token_indices, int32_t* offsets,
                                               int32_t* kept_counts, float* aux_loss,
                                               void* permuted, float* routing_w,
                                               int32_t* source_idx, int32_t* slot_pos,
                                               int32_t* err, lr_stream_t stream) {
  if (T <= 0 || E < 1 || E > 64 || k < 1 || k > kMaxTopK || k > E || capacity < 1)
    return LR_ERR_INVALID_ARGUMENT;
  const int B = (T + kRouteThreads - 1) / kRouteThreads;
  if (route_ws_bytes_for(B, E, true) > kStaticRouteScratchBytes) return LR_ERR_TOO_LARGE;
  void* scratch = nullptr;
  const int rc = route_scratch_address(&scratch);
  if (rc != LR_OK) return rc;
  // The shared ticket word is cleared on the stream by the dispatch itself;
  // the per-block counts, bases and sums are fully rewritten by every call.
  return lr_topk_gating_dispatch(x, logits, T, d, E, k, capacity, load_balance_weight,
                                 fill_dropped, expert_ids, gate_weights, token_indices, offsets,
                                 kept_counts, aux_loss, permuted, routing_w, source_idx, slot_pos,
                                 scratch, kStaticRouteScratchBytes, err, stream);
}
