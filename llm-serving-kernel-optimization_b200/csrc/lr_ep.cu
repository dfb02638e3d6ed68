// lr_ep.cu -- expert-parallel token exchange over NVLink peer memory (one process per GPU).
//
// The exchange the reference serving worker would need between its GPUs
// (lightning_router/serving/worker.py:156-186 runs every expert on every GPU
// instead) done without a host round trip:
//   * every rank keeps its tokens, the row -> token map of its uncapped expert
//     segments and its expert outputs in buffers the other ranks have mapped
//     (CUDA IPC, plain peer loads over NVLink; no NVLS or multimem objects);
//   * lr_ep_plan turns the all-gathered per-(rank, expert) counts into the
//     global slot-order capacity decision and both sides' row layouts, on the
//     device;
//   * lr_ep_gather (expert owner) pulls the kept token rows of its experts from
//     their source ranks into its own [expert][source rank] segments, the
//     layout the grouped GEMM reads;
//   * lr_ep_combine (token owner) pulls each kept slot's expert output row from
//     the expert owner and sums them in slot order in fp32, exactly as the
//     single-GPU combine.
// Cross-rank ordering needs no collective library call in the step: flags in
// the mapped memory, written with release and read with acquire semantics at
// system scope, with every wait bounded in time (LR_DEVERR_PEER_TIMEOUT):
//   * lr_ep_publish writes this rank's statistics row (token count, per-expert
//     counts and probability sums) into every rank's table and raises its
//     "stats" flag there; lr_ep_plan_wait waits for every rank's flag of the
//     step, then plans and computes the auxiliary loss;
//   * lr_ep_signal raises this rank's "outputs" flag on every rank after its
//     expert GEMMs; lr_ep_combine waits for every rank's flag before it reads.
// Flags hold the step number (the epoch), so nothing is reset between steps.
// A rank overwrites its token and row-map buffers only after its combine saw
// every owner's outputs flag (so every owner's gather of the previous step is
// done), and an owner overwrites its outputs only after its plan saw every
// rank's stats flag of the next step (so every combine of the previous step is
// done).  Publish and wait are separate launches, so ranks emulated one after
// the other on one GPU never wait on a later launch.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "lr_common.cuh"

namespace lr {

constexpr int kEpMaxCounts = 4096;  // G * E entries handled by the plan kernel

struct EpPlanLayout {
  int El, seg_start, seg_len, row_base, src_off, kept, my_off, my_kept, dst_row, cap, total;
  __host__ __device__ EpPlanLayout(int G, int E) {
    El = E / G;
    seg_start = 0;
    seg_len = El;
    row_base = 2 * El;
    src_off = row_base + El * G;
    kept = src_off + El * G;
    my_off = kept + El * G;
    my_kept = my_off + E;
    dst_row = my_kept + E;
    cap = dst_row + E;  // the capacity the plan applied
    total = cap + 1;
  }
};

// Plan of one rank, one block, from s_cnt[r*E + e] = slots of expert e on rank r
// (uncapped, in the rank's slot order) and the capacity C.  Rank r's slots of e
// follow those of lower ranks in the global slot order, so kept(r, e) =
// clamp(C - sum_{r' < r} counts[r'][e], 0, counts[r][e]) -- the single-GPU
// capacity rule.
LR_DEVICE void ep_plan_block(const int* s_cnt, int* s_kept, int G, int E, int rank, int C,
                             int32_t* __restrict__ plan) {
  const EpPlanLayout L(G, E);
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int base = 0;
    for (int r = 0; r < G; ++r) {
      const int c = s_cnt[r * E + e];
      const int k = C - base;
      s_kept[r * E + e] = k < 0 ? 0 : (k > c ? c : k);
      base += c;
    }
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  plan[L.cap] = C;
  const int El = L.El;
  // owner side: segments [local expert][source rank]
  int row = 0;
  for (int el = 0; el < El; ++el) {
    const int e = rank * El + el;
    plan[L.seg_start + el] = row;
    int len = 0;
    for (int r = 0; r < G; ++r) {
      int off = 0;
      for (int e2 = 0; e2 < e; ++e2) off += s_cnt[r * E + e2];
      const int kp = s_kept[r * E + e];
      plan[L.row_base + el * G + r] = row + len;
      plan[L.src_off + el * G + r] = off;
      plan[L.kept + el * G + r] = kp;
      len += kp;
    }
    plan[L.seg_len + el] = len;
    row += len;
  }
  // source side: this rank's segments and where its kept rows land at each owner
  int off = 0;
  for (int e = 0; e < E; ++e) {
    plan[L.my_off + e] = off;
    off += s_cnt[rank * E + e];
    plan[L.my_kept + e] = s_kept[rank * E + e];
    const int o = e / El, el = e % El;
    int start = 0;
    for (int e2 = o * El; e2 < o * El + el; ++e2)
      for (int r = 0; r < G; ++r) start += s_kept[r * E + e2];
    for (int r = 0; r < rank; ++r) start += s_kept[r * E + e];
    plan[L.dst_row + e] = start;
  }
}

// C = max(int((k * T / E) * cf), 1) in double precision, as on one GPU
// (reference kernels/expert_routing.py:196-197), clipped to the buffers' bound.
LR_DEVICE int ep_capacity(long long T, int top_k, int E, double cf, int cap_max, int32_t* err) {
  const double q = double(T * top_k) / double(E);
  const long long c = (long long)(q * cf);
  if (c > cap_max) report(err, LR_DEVERR_BAD_SEGMENT);  // buffers too small: rows clipped
  return c < 1 ? 1 : (c > cap_max ? cap_max : int(c));
}

// One block.  counts[r*E + e] from the caller.  With shard_tokens (the G ranks'
// token counts) the capacity is computed as on one GPU, `capacity` being the
// largest C the caller's buffers hold; otherwise C = capacity.
__global__ void __launch_bounds__(256)
    ep_plan_kernel(const int32_t* __restrict__ counts, const int32_t* __restrict__ shard_tokens,
                   int G, int E, int top_k, double cf, int rank, int capacity,
                   int32_t* __restrict__ plan, int32_t* err) {
  __shared__ int s_cnt[kEpMaxCounts];
  __shared__ int s_kept[kEpMaxCounts];
  __shared__ int s_cap;
  for (int i = threadIdx.x; i < G * E; i += blockDim.x) {
    int c = counts[i];
    if (c < 0) {
      report(err, LR_DEVERR_BAD_SEGMENT);
      c = 0;
    }
    s_cnt[i] = c;
  }
  if (threadIdx.x == 0) {
    int C = capacity;
    if (shard_tokens) {
      long long T = 0;
      for (int r = 0; r < G; ++r) {
        const int t = shard_tokens[r];
        if (t < 0) report(err, LR_DEVERR_BAD_SEGMENT);
        else T += t;
      }
      C = ep_capacity(T, top_k, E, cf, capacity, err);
    }
    s_cap = C;
  }
  __syncthreads();
  ep_plan_block(s_cnt, s_kept, G, E, rank, s_cap, plan);
}

LR_DEVICE void st_release_sys(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
LR_DEVICE int32_t ld_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

constexpr uint64_t kPeerWaitNs = 5000000000ull;  // 5 s: a rank that far behind has failed

// Waits until flags[i] >= epoch for i < n; false (and LR_DEVERR_PEER_TIMEOUT) when
// one has not arrived within kPeerWaitNs.
LR_DEVICE bool wait_flags(const int32_t* flags, int n, int epoch, int32_t* err) {
  const uint64_t t0 = global_timer_ns();
  for (int i = 0; i < n; ++i) {
    while (ld_acquire_sys(flags + i) < epoch) {
      if (global_timer_ns() - t0 > kPeerWaitNs) {
        report(err, LR_DEVERR_PEER_TIMEOUT);
        return false;
      }
    }
  }
  return true;
}

// This rank's statistics row [T, count[0..E), prob_sum[0..E)] (doubles) into
// slot `rank` of every rank's table, then this rank's stats flag on every rank.
__global__ void __launch_bounds__(256)
    ep_publish_kernel(const uint64_t* __restrict__ peer_stats,
                      const uint64_t* __restrict__ peer_flags, const int32_t* __restrict__ offsets,
                      const double* __restrict__ prob_sums, int T_l, int G, int E, int rank,
                      int epoch) {
  const int W = 1 + 2 * E;
  for (int i = threadIdx.x; i < G * W; i += blockDim.x) {
    const int q = i / W, j = i % W;
    double v = 0.0;
    if (j == 0) v = double(T_l);
    else if (offsets && j <= E) v = double(offsets[j] - offsets[j - 1]);
    else if (prob_sums && j > E) v = prob_sums[j - 1 - E];
    reinterpret_cast<double*>(peer_stats[q])[rank * W + j] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int q = 0; q < G; ++q) st_release_sys(reinterpret_cast<int32_t*>(peer_flags[q]) + rank, epoch);
  }
}

// Waits for every rank's stats row of step `epoch` in this rank's table, then
// plans (ep_plan_block) and writes the auxiliary loss of the whole job,
// lbw * E * sum_e f_e P_e with f_e = count_e / (k T), P_e = prob_sum_e / T
// (reference lightning_router/models/gating.py:91-99).  When a flag does not
// arrive the plan keeps no rows.
__global__ void __launch_bounds__(256)
    ep_plan_wait_kernel(const double* __restrict__ stats, const int32_t* __restrict__ flags,
                        int G, int E, int rank, int top_k, double cf, int cap_max, float lbw,
                        int epoch, int32_t* __restrict__ plan, float* __restrict__ aux,
                        int32_t* err) {
  __shared__ int s_cnt[kEpMaxCounts];
  __shared__ int s_kept[kEpMaxCounts];
  __shared__ int s_ok, s_cap;
  if (threadIdx.x == 0) s_ok = wait_flags(flags, G, epoch, err) ? 1 : 0;
  __syncthreads();
  const int W = 1 + 2 * E;
  for (int i = threadIdx.x; i < G * E; i += blockDim.x) {
    const int r = i / E, e = i % E;
    const double c = s_ok ? __ldcv(stats + r * W + 1 + e) : 0.0;
    s_cnt[i] = c > 0.0 ? int(c + 0.5) : 0;
  }
  if (threadIdx.x == 0) {
    double T = 0.0;
    for (int r = 0; r < G; ++r) T += s_ok ? __ldcv(stats + r * W) : 0.0;
    s_cap = ep_capacity((long long)(T + 0.5), top_k, E, cf, cap_max, err);
    double a = 0.0;
    if (s_ok && T > 0.0) {
      for (int e = 0; e < E; ++e) {
        double cnt = 0.0, ps = 0.0;
        for (int r = 0; r < G; ++r) {
          cnt += __ldcv(stats + r * W + 1 + e);
          ps += __ldcv(stats + r * W + 1 + E + e);
        }
        a += (cnt / (T * top_k)) * (ps / T);
      }
    }
    *aux = float(double(lbw) * E * a);
  }
  __syncthreads();
  ep_plan_block(s_cnt, s_kept, G, E, rank, s_cap, plan);
}

// This rank's outputs flag (slot `rank` of the second half) on every rank.
__global__ void ep_signal_kernel(const uint64_t* __restrict__ peer_flags, int G, int rank,
                                 int epoch) {
  if (threadIdx.x != 0) return;
  __threadfence_system();
  for (int q = 0; q < G; ++q)
    st_release_sys(reinterpret_cast<int32_t*>(peer_flags[q]) + G + rank, epoch);
}

// Peer read of a 16-byte vector (plain global load: the data is stable while
// the kernel runs, and it may live on another GPU).
LR_DEVICE uint4 ld_peer(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

constexpr int kEpUnroll = 8;

// Owner side: one warp per destination row.
__global__ void __launch_bounds__(256)
    ep_gather_kernel(const uint64_t* __restrict__ peer_x, const uint64_t* __restrict__ peer_src,
                     const int32_t* __restrict__ plan, int G, int E, int rank, int T_max,
                     int S_max, int d8, int rows_max, uint4* __restrict__ out, int32_t* err) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows_max) return;
  const int lane = threadIdx.x & 31;
  const EpPlanLayout L(G, E);
  const int n = L.El * G;
  int found = -1;
  for (int i = lane; i < n; i += 32) {
    const int rb = __ldg(plan + L.row_base + i), kp = __ldg(plan + L.kept + i);
    if (row >= rb && row < rb + kp) found = i;
  }
  found = __reduce_max_sync(0xffffffffu, found);
  if (found < 0) return;  // beyond the kept rows: never read by the GEMM
  const int r = found % G;
  const int idx = __ldg(plan + L.src_off + found) + (row - __ldg(plan + L.row_base + found));
  int t = -1;
  if (lane == 0 && idx >= 0 && idx < S_max)
    t = reinterpret_cast<const int32_t*>(peer_src[r])[idx];
  t = __shfl_sync(0xffffffffu, t, 0);
  if (t < 0 || t >= T_max) {
    if (lane == 0) report(err, LR_DEVERR_BAD_TOKEN);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(peer_x[r]) + size_t(t) * d8;
  uint4* dst = out + size_t(row) * d8;
  for (int c0 = 0; c0 < d8; c0 += 32 * kEpUnroll) {
    uint4 v[kEpUnroll];
#pragma unroll
    for (int u = 0; u < kEpUnroll; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < d8) v[u] = ld_peer(src + c);
    }
#pragma unroll
    for (int u = 0; u < kEpUnroll; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < d8) dst[c] = v[u];
    }
  }
}

constexpr int kEpCombUnroll = 4;

// Token-owner side: one warp per token, its kept slots' output rows pulled from
// the expert owners and summed in slot order (fp32 FMA, one fp16 rounding).
__global__ void __launch_bounds__(256)
    ep_combine_kernel(const uint64_t* __restrict__ peer_y, const int32_t* __restrict__ plan,
                      const int32_t* __restrict__ expert_ids, const float* __restrict__ gate_w,
                      const int32_t* __restrict__ slot_pos, int T, int k, int G, int E, int d8,
                      int rows_max, uint4* __restrict__ out, int32_t* err,
                      const int32_t* __restrict__ ready, int epoch) {
  if (ready) {
    // every owner's outputs of this step are written (and every owner's gather
    // of this step has read this rank's tokens)
    __shared__ int s_ok;
    if (threadIdx.x == 0) s_ok = wait_flags(ready, G, epoch, err) ? 1 : 0;
    __syncthreads();
    if (!s_ok) return;
  }
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  const EpPlanLayout L(G, E);
  int my_o = -1, my_row = 0;
  float my_w = 0.f;
  if (lane < k) {
    const size_t s = size_t(t) * k + lane;
    const int e = __ldg(expert_ids + s);
    if (e >= 0 && e < E) {
      const int rk = __ldg(slot_pos + s) - __ldg(plan + L.my_off + e);
      if (rk >= 0 && rk < __ldg(plan + L.my_kept + e)) {
        const int row = __ldg(plan + L.dst_row + e) + rk;
        if (row < rows_max) {
          my_o = e / L.El;
          my_row = row;
          my_w = __ldg(gate_w + s);
        } else {
          report(err, LR_DEVERR_BAD_SEGMENT);
        }
      }
    } else {
      report(err, LR_DEVERR_BAD_EXPERT);
    }
  }
  int o[kMaxTopK], rows[kMaxTopK];
  float w[kMaxTopK];
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    o[j] = __shfl_sync(0xffffffffu, my_o, j);
    rows[j] = __shfl_sync(0xffffffffu, my_row, j);
    w[j] = __shfl_sync(0xffffffffu, my_w, j);
  }
  for (int c0 = 0; c0 < d8; c0 += 32 * kEpCombUnroll) {
    float acc[kEpCombUnroll][8];
#pragma unroll
    for (int u = 0; u < kEpCombUnroll; ++u)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[u][i] = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) {
      if (j < k && o[j] >= 0) {
        const uint4* row = reinterpret_cast<const uint4*>(peer_y[o[j]]) + size_t(rows[j]) * d8;
        uint4 v[kEpCombUnroll];
#pragma unroll
        for (int u = 0; u < kEpCombUnroll; ++u) {
          const int c = c0 + u * 32 + lane;
          if (c < d8) v[u] = ld_peer(row + c);
        }
#pragma unroll
        for (int u = 0; u < kEpCombUnroll; ++u) {
          const int c = c0 + u * 32 + lane;
          if (c < d8) acc_half8(acc[u], v[u], w[j]);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kEpCombUnroll; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < d8) out[size_t(t) * d8 + c] = pack_half8(acc[u]);
    }
  }
}

static PFN_cuMemGetAddressRange_v3020 get_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  }
  return fn;
}

}  // namespace lr

using namespace lr;

extern "C" int lr_ep_plan_size(int world, int num_experts) {
  if (world < 1 || num_experts < 1 || num_experts % world) return 0;
  return EpPlanLayout(world, num_experts).total;
}

extern "C" int lr_ep_plan(const int32_t* counts, int world, int num_experts, int rank,
                          int capacity, int32_t* plan, int32_t* err, lr_stream_t stream) {
  if (!counts || !plan || world < 1 || num_experts < 1 || num_experts % world ||
      rank < 0 || rank >= world || capacity < 1 || world * num_experts > kEpMaxCounts)
    return LR_ERR_INVALID_ARGUMENT;
  ep_plan_kernel<<<1, 256, 0, stream>>>(counts, nullptr, world, num_experts, 1, 1.0, rank,
                                        capacity, plan, err);
  LR_LAUNCH_CHECK();
  return LR_OK;
}

extern "C" int lr_ep_plan_tokens(const int32_t* counts, const int32_t* shard_tokens, int world,
                                 int num_experts, int top_k, double capacity_factor, int rank,
                                 int max_capacity, int32_t* plan, int32_t* err,
                                 lr_stream_t stream) {
  if (!counts || !shard_tokens || !plan || world < 1 || num_experts < 1 ||
      num_experts % world || rank < 0 || rank >= world || top_k < 1 || !(capacity_factor > 0) ||
      max_capacity < 1 || world * num_experts > kEpMaxCounts)
    return LR_ERR_INVALID_ARGUMENT;
  ep_plan_kernel<<<1, 256, 0, stream>>>(counts, shard_tokens, world, num_experts, top_k,
                                        capacity_factor, rank, max_capacity, plan, err);
  LR_LAUNCH_CHECK();
  return LR_OK;
}

extern "C" int lr_ep_gather(const uint64_t* peer_x, const uint64_t* peer_src, const int32_t* plan,
                            int world, int num_experts, int rank, int max_tokens, int max_slots,
                            int d, int rows_max, void* out, int32_t* err, lr_stream_t stream) {
  if (!peer_x || !peer_src || !plan || !out || world < 1 || num_experts % world || rank < 0 ||
      rank >= world || d <= 0 || d % 8 || rows_max < 0 || max_tokens < 0 || max_slots < 0 ||
      (reinterpret_cast<uintptr_t>(out) & 15u))
    return LR_ERR_INVALID_ARGUMENT;
  if (rows_max == 0) return LR_OK;
  ep_gather_kernel<<<(rows_max + 7) / 8, 256, 0, stream>>>(
      peer_x, peer_src, plan, world, num_experts, rank, max_tokens, max_slots, d / 8, rows_max,
      static_cast<uint4*>(out), err);
  LR_LAUNCH_CHECK();
  return LR_OK;
}

extern "C" int lr_ep_publish(const uint64_t* peer_stats, const uint64_t* peer_flags,
                             const int32_t* offsets, const double* prob_sums, int num_tokens,
                             int world, int num_experts, int rank, int epoch, lr_stream_t stream) {
  if (!peer_stats || !peer_flags || world < 1 || num_experts < 1 || rank < 0 || rank >= world ||
      num_tokens < 0 || epoch < 1 || (num_tokens > 0 && (!offsets || !prob_sums)))
    return LR_ERR_INVALID_ARGUMENT;
  ep_publish_kernel<<<1, 256, 0, stream>>>(peer_stats, peer_flags, offsets, prob_sums, num_tokens,
                                           world, num_experts, rank, epoch);
  LR_LAUNCH_CHECK();
  return LR_OK;
}

extern "C" int lr_ep_plan_wait(const double* stats, const int32_t* flags, int world,
                               int num_experts, int rank, int top_k, double capacity_factor,
                               int max_capacity, float load_balance_weight, int epoch,
                               int32_t* plan, float* aux_loss, int32_t* err, lr_stream_t stream) {
  if (!stats || !flags || !plan || !aux_loss || world < 1 || num_experts < 1 ||
      num_experts % world || rank < 0 || rank >= world || top_k < 1 ||
      !(capacity_factor > 0) || max_capacity < 1 || epoch < 1 ||
      world * num_experts > kEpMaxCounts)
    return LR_ERR_INVALID_ARGUMENT;
  ep_plan_wait_kernel<<<1, 256, 0, stream>>>(stats, flags, world, num_experts, rank, top_k,
                                             capacity_factor, max_capacity, load_balance_weight,
                                             epoch, plan, aux_loss, err);
  LR_LAUNCH_CHECK();
  return LR_OK;
}

extern "C" int lr_ep_signal(const uint64_t* peer_flags, int world, int rank, int epoch,
                            lr_stream_t stream) {
  if (!peer_flags || world < 1 || rank < 0 || rank >= world || epoch < 1)
    return LR_ERR_INVALID_ARGUMENT;
  ep_signal_kernel<<<1, 32, 0, stream>>>(peer_flags, world, rank, epoch);
  LR_LAUNCH_CHECK();
  return LR_OK;
}

extern "C" int lr_ep_combine(const uint64_t* peer_y, const int32_t* plan,
                             const int32_t* expert_ids, const float* gate_weights,
                             const int32_t* slot_pos, int T, int k, int world, int num_experts,
                             int d, int rows_max, void* out, const int32_t* ready_flags,
                             int epoch, int32_t* err, lr_stream_t stream) {
  if (!peer_y || !plan || !expert_ids || !gate_weights || !slot_pos || !out || T < 0 || k < 1 ||
      k > kMaxTopK || world < 1 || num_experts % world || d <= 0 || d % 8 ||
      (reinterpret_cast<uintptr_t>(out) & 15u))
    return LR_ERR_INVALID_ARGUMENT;
  if (T == 0) return LR_OK;
  if (ready_flags && epoch < 1) return LR_ERR_INVALID_ARGUMENT;
  ep_combine_kernel<<<(T + 7) / 8, 256, 0, stream>>>(peer_y, plan, expert_ids, gate_weights,
                                                     slot_pos, T, k, world, num_experts, d / 8,
                                                     rows_max, static_cast<uint4*>(out), err,
                                                     ready_flags, epoch);
  LR_LAUNCH_CHECK();
  return LR_OK;
}

extern "C" int lr_ipc_export(const void* ptr, void* handle, uint64_t* offset) {
  if (!ptr || !handle || !offset) return LR_ERR_INVALID_ARGUMENT;
  auto fn = get_range_fn();
  if (!fn) return LR_ERR_NO_DEVICE;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return LR_ERR_INVALID_ARGUMENT;
  LR_CUDA_TRY(cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle),
                                  reinterpret_cast<void*>(base)));
  *offset = uint64_t(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return LR_OK;
}

extern "C" int lr_ipc_import(const void* handle, uint64_t offset, void** ptr, void** base) {
  if (!handle || !ptr || !base) return LR_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  LR_CUDA_TRY(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr = static_cast<char*>(*base) + offset;
  return LR_OK;
}

extern "C" int lr_ipc_close(void* base) {
  if (!base) return LR_ERR_INVALID_ARGUMENT;
  LR_CUDA_TRY(cudaIpcCloseMemHandle(base));
  return LR_OK;
}
