// DeepSeek-V3 no-aux routing and the token permutation that follows it.
//
// route_kernel      one warp per token (reference: noaux_routing_topk8_kernel,
//                   solution/cuda/kernel.cu:2278-2375, which uses one CTA of
//                   256 threads per token and a serial thread-0 selection).
// permute_kernel    deterministic per-expert segments without a host sync
//                   (reference: count/compute_offsets/fill kernels,
//                   solution/cuda/kernel.cu:86-100 and 2465-2495, whose fill
//                   order inside a segment depends on atomics).
#include <cuda_bf16.h>
#include <cstdint>

#include "hidden_quant.cuh"
#include "moe_kernels.cuh"
#include "moe_ptx.cuh"
#include "moe_shapes.cuh"

namespace moe {

namespace {

// Total order used for every top-k in routing: larger value first, and on
// equal values the smaller expert index first.
__device__ __forceinline__ bool ranks_before(float va, int ia, float vb, int ib) {
  return (va > vb) || (va == vb && ia < ib);
}

// Unsigned key with the order of the float values (for non-NaN inputs; -0.0
// cannot occur here since scores are strictly positive).
__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

}  // namespace

// Routes token t with one warp: lane l owns experts 8l .. 8l+7, so group g
// (32 experts) is owned by lanes 4g .. 4g+3.
// Lanes 0..7 return the token's k-th selection (expert id and weight) in
// out_idx / out_w and also store them to topk_idx / topk_w.
__device__ __forceinline__ void route_token(const RouteParams& p, int t, int lane, int& out_idx,
                                            float& out_w) {

  // ---- scores -------------------------------------------------------------
  const float4* lrow = reinterpret_cast<const float4*>(p.logits + static_cast<int64_t>(t) * kExpertsGlobal);
  float4 l0 = lrow[2 * lane];
  float4 l1 = lrow[2 * lane + 1];
  float x[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
  float b[8];
  if (p.bias_is_fp32) {
    const float4* brow = reinterpret_cast<const float4*>(p.bias);
    float4 b0 = brow[2 * lane];
    float4 b1 = brow[2 * lane + 1];
    b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
    b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
  } else {
    const uint4 raw = reinterpret_cast<const uint4*>(p.bias)[lane];
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      b[2 * j] = __uint_as_float(w[j] << 16);
      b[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  }
  float s[8], sb[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    s[j] = 1.0f / (1.0f + expf(-x[j]));   // accurate expf and IEEE division
    sb[j] = s[j] + b[j];
  }

  // ---- group score: sum of the two largest biased scores ------------------
  float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float v = sb[j];
    if (v > m1) { m2 = m1; m1 = v; }
    else if (v > m2) { m2 = v; }
  }
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    const float o1 = __shfl_xor_sync(0xffffffffu, m1, off);
    const float o2 = __shfl_xor_sync(0xffffffffu, m2, off);
    const float n1 = fmaxf(m1, o1);
    const float n2 = fmaxf(fminf(m1, o1), fmaxf(m2, o2));
    m1 = n1;
    m2 = n2;
  }
  const float my_group_score = m1 + m2;
  const int my_group = lane >> 2;
  int rank = 0;
#pragma unroll
  for (int g = 0; g < kGroups; ++g) {
    const float gs = __shfl_sync(0xffffffffu, my_group_score, 4 * g);
    rank += ranks_before(gs, g, my_group_score, my_group) ? 1 : 0;
  }
  const bool keep = rank < kTopKGroups;

  // ---- the 128 candidates of the 4 kept groups, 4 per lane ------------------
  // Lane L takes experts 32g + 4(L & 7) .. +3 of the (L >> 3)-th kept group g
  // in increasing group order (owned by lane 4g + (L & 7) / 2, its elements
  // 4(L & 1) .. +3), so lane order is still expert order and every lane has
  // half the candidates to scan in each selection round.
  const uint32_t kept = __ballot_sync(0xffffffffu, keep && (lane & 3) == 0);   // bit 4g per kept group
  const int cg = static_cast<int>(__fns(kept, 0u, (lane >> 3) + 1)) >> 2;
  const int src = 4 * cg + ((lane & 7) >> 1);
  const bool upper = lane & 1;
  float cand[4], cs[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float vl = __shfl_sync(0xffffffffu, sb[i], src);
    const float vh = __shfl_sync(0xffffffffu, sb[4 + i], src);
    const float sl = __shfl_sync(0xffffffffu, s[i], src);
    const float sh = __shfl_sync(0xffffffffu, s[4 + i], src);
    cand[i] = upper ? vh : vl;
    cs[i] = upper ? sh : sl;
  }
  const int cand0 = 32 * cg + 4 * (lane & 7);   // expert of cand[0]

  // ---- top-8 experts among the kept groups --------------------------------
  // Each round takes the largest remaining candidate: every lane offers its
  // best untaken one (lowest index on equal values), one warp max over an
  // order-preserving integer key finds the value, and the lowest lane
  // offering it wins -- lanes hold increasing expert ranges, so that is the
  // lowest expert index among equal values, the same total order as
  // ranks_before.
  uint32_t taken = 0;
  int sel_idx[kTopK];
  float sel_s[kTopK];
#pragma unroll
  for (int k = 0; k < kTopK; ++k) {
    float bv = -INFINITY;
    int bj = -1;
    float bs = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (!((taken >> j) & 1u) && (bj < 0 || cand[j] > bv)) {
        bv = cand[j];
        bj = j;
        bs = cs[j];
      }
    }
    // a candidate's key is at least 1, so it always beats a lane with none
    // left (key 0), even when its value is the NaN whose order key is 0
    const uint32_t key = bj >= 0 ? max(order_key(bv), 1u) : 0u;
    const uint32_t best = __reduce_max_sync(0xffffffffu, key);
    const int wl = __ffs(__ballot_sync(0xffffffffu, key == best)) - 1;
    if (lane == wl) taken |= 1u << bj;
    sel_idx[k] = __shfl_sync(0xffffffffu, cand0 + bj, wl);
    sel_s[k] = __shfl_sync(0xffffffffu, bs, wl);
  }

  // ---- weights: unbiased scores renormalised over the selection ------------
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < kTopK; ++k) sum += sel_s[k];
  sum = fmaxf(sum, 1e-20f);
  int my_idx = sel_idx[0];
  float my_s = sel_s[0];
#pragma unroll
  for (int k = 1; k < kTopK; ++k) {
    if (lane == k) { my_idx = sel_idx[k]; my_s = sel_s[k]; }
  }
  out_idx = my_idx;
  out_w = (my_s / sum) * p.routed_scaling_factor;
  if (lane < kTopK) {
    p.topk_idx[t * kTopK + lane] = out_idx;
    p.topk_w[t * kTopK + lane] = out_w;
  }
}

// The other routing methods of this operator family, restated from the
// published reference functions of flashinfer's MoE trace templates
// (flashinfer/trace/templates/moe.py: default 187-225, renormalize 227-266,
// llama4 268-307, renormalize_naive 309-349, topk 351-390). With
// l = logit + bias (no bias: l = logit):
//   Default           top-k of softmax(l)   w = softmax(l)[e]
//   Renormalize       top-k of l            w = softmax of l over the picks
//   Llama4            top-1 of l            w = sigmoid(l[e])
//   RenormalizeNaive  top-k of softmax(l)   w = softmax(l)[e] / (sum over picks + 1e-20)
//   TopK              top-k of l            w = 1 / k
// each weight times routed_scaling_factor (TopK: routed_scaling_factor / k).
// Softmax is monotonic, so every method selects by l, in the total order of
// all routing here (larger first, smaller expert id on equal values; -0.0
// counts as 0.0). Lane l owns experts 8l .. 8l+7 as in route_token; lanes
// 0..7 return and store selection k, with kNoExpert and weight 0 in the
// slots k >= top_k.
__device__ __forceinline__ void route_token_simple(const RouteParams& p, int t, int lane, int& out_idx,
                                                   float& out_w) {
  const float4* lrow = reinterpret_cast<const float4*>(p.logits + static_cast<int64_t>(t) * kExpertsGlobal);
  const float4 l0 = lrow[2 * lane];
  const float4 l1 = lrow[2 * lane + 1];
  float l[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
  if (p.bias != nullptr) {
    if (p.bias_is_fp32) {
      const float4* brow = reinterpret_cast<const float4*>(p.bias);
      const float4 b0 = brow[2 * lane];
      const float4 b1 = brow[2 * lane + 1];
      const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) l[j] += b[j];
    } else {
      const uint4 raw = reinterpret_cast<const uint4*>(p.bias)[lane];
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        l[2 * j] += __uint_as_float(w[j] << 16);
        l[2 * j + 1] += __uint_as_float(w[j] & 0xFFFF0000u);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j)   // -0.0 -> +0.0: equal values, one key
    if (__float_as_uint(l[j]) == 0x80000000u) l[j] = 0.0f;

  // ---- top-k: per round the lane's best untaken expert, then the warp's --
  const int K = p.top_k;
  uint32_t taken = 0;
  int sel_idx[kTopK];
  float sel_l[kTopK];
#pragma unroll
  for (int k = 0; k < kTopK; ++k) {
    sel_idx[k] = kNoExpert;
    sel_l[k] = 0.f;
    if (k < K) {
      uint32_t bk = 0;
      int bj = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        // untaken experts have keys >= 1 (the NaN whose order key is 0
        // included), so a taken one (key 0) is never picked again
        const uint32_t key = ((taken >> j) & 1u) ? 0u : max(order_key(l[j]), 1u);
        if (key > bk) {
          bk = key;
          bj = j;
        }
      }
      const uint32_t wk = __reduce_max_sync(0xffffffffu, bk);
      const int wl = __ffs(__ballot_sync(0xffffffffu, bk == wk)) - 1;
      const int wj = __shfl_sync(0xffffffffu, bj, wl);
      float lv = l[0];
#pragma unroll
      for (int j = 1; j < 8; ++j) lv = (j == bj) ? l[j] : lv;
      sel_l[k] = __shfl_sync(0xffffffffu, lv, wl);
      sel_idx[k] = 8 * wl + wj;
      if (lane == wl) taken |= 1u << wj;
    }
  }

  // ---- weights --------------------------------------------------------------
  float wsel[kTopK];
  const int m = p.method;
  if (m == kRouteDefault || m == kRouteRenormalizeNaive) {
    float mx = l[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) mx = fmaxf(mx, l[j]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float z = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) z += expf(l[j] - mx);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) z += __shfl_xor_sync(0xffffffffu, z, off);
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
      wsel[k] = k < K ? expf(sel_l[k] - mx) / z : 0.f;
      sum += wsel[k];
    }
    if (m == kRouteRenormalizeNaive) {
#pragma unroll
      for (int k = 0; k < kTopK; ++k) wsel[k] = wsel[k] / (sum + 1e-20f);
    }
#pragma unroll
    for (int k = 0; k < kTopK; ++k) wsel[k] *= p.routed_scaling_factor;
  } else if (m == kRouteRenormalize) {
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
      wsel[k] = k < K ? expf(sel_l[k] - sel_l[0]) : 0.f;
      sum += wsel[k];
    }
#pragma unroll
    for (int k = 0; k < kTopK; ++k) wsel[k] = wsel[k] / sum * p.routed_scaling_factor;
  } else if (m == kRouteLlama4) {
#pragma unroll
    for (int k = 0; k < kTopK; ++k)
      wsel[k] = k == 0 ? 1.0f / (1.0f + expf(-sel_l[0])) * p.routed_scaling_factor : 0.f;
  } else {   // kRouteTopK
#pragma unroll
    for (int k = 0; k < kTopK; ++k) wsel[k] = k < K ? p.routed_scaling_factor / static_cast<float>(K) : 0.f;
  }

  int my_idx = kNoExpert;
  float my_w = 0.f;
#pragma unroll
  for (int k = 0; k < kTopK; ++k) {
    if (lane == k) {
      my_idx = sel_idx[k];
      my_w = wsel[k];
    }
  }
  out_idx = my_idx;
  out_w = my_w;
  if (lane < kTopK) {
    p.topk_idx[t * kTopK + lane] = my_idx;
    p.topk_w[t * kTopK + lane] = my_w;
  }
}

// Selections given by the caller (kRouteGiven): lane k < top_k takes entry
// k of token t as it is; the other slots hold kNoExpert and weight 0. No
// logits are read and no scaling factor is applied.
__device__ __forceinline__ void route_token_given(const RouteParams& p, int t, int lane, int& out_idx,
                                                  float& out_w) {
  int idx = kNoExpert;
  float w = 0.f;
  if (lane < p.top_k) {
    idx = __ldg(p.given_idx + static_cast<int64_t>(t) * p.top_k + lane);
    w = __ldg(p.given_w + static_cast<int64_t>(t) * p.top_k + lane);
  }
  out_idx = idx;
  out_w = w;
  if (lane < kTopK) {
    p.topk_idx[t * kTopK + lane] = idx;
    p.topk_w[t * kTopK + lane] = w;
  }
}

__device__ __forceinline__ void route_token_any(const RouteParams& p, int t, int lane, int& out_idx, float& out_w) {
  if (p.method == kRouteDeepSeekV3)
    route_token(p, t, lane, out_idx, out_w);
  else if (p.method == kRouteGiven)
    route_token_given(p, t, lane, out_idx, out_w);
  else
    route_token_simple(p, t, lane, out_idx, out_w);
}

// One warp per token, 8 tokens per CTA.
__global__ void __launch_bounds__(256) route_kernel(RouteParams p) {
  pdl_launch_next();
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  int idx;
  float w;
  if (t >= p.num_tokens) return;
  route_token_any(p, t, lane, idx, w);
  // A token with no pick among the local experts gets no combine row, so its
  // output row is zero: written here, where the stores overlap the routing
  // arithmetic of the other warps, and skipped by finalize_kernel.
  const bool local = lane < kTopK && static_cast<unsigned>(idx - p.local_expert_offset) < kExpertsLocal;
  if (p.out != nullptr && !__any_sync(0xffffffffu, local)) {
    uint4* orow = reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(t) * kHidden);
#pragma unroll
    for (int i = 0; i < kHidden / 8 / 32; ++i) orow[lane + 32 * i] = make_uint4(0u, 0u, 0u, 0u);
  }
}

namespace {

// The local-expert selections of token t as a 32-bit mask (bit e = local
// expert e) with the (local id, weight) pairs in routing order.
__device__ __forceinline__ uint32_t token_selection(const PermuteParams& p, int t, int (&sidx)[kTopK],
                                                    float (&sw)[kTopK]) {
  uint32_t mask = 0;
  if (t < p.num_tokens) {
    const int4* ip = reinterpret_cast<const int4*>(p.topk_idx + t * kTopK);
    const float4* wp = reinterpret_cast<const float4*>(p.topk_w + t * kTopK);
    const int4 i0 = ip[0], i1 = ip[1];
    const float4 w0 = wp[0], w1 = wp[1];
    const int ii[8] = {i0.x, i0.y, i0.z, i0.w, i1.x, i1.y, i1.z, i1.w};
    const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
      const int le = ii[k] - p.local_expert_offset;
      sidx[k] = le;
      sw[k] = ww[k];
      if (le >= 0 && le < kExpertsLocal) mask |= 1u << le;
    }
  } else {
#pragma unroll
    for (int k = 0; k < kTopK; ++k) { sidx[k] = -1; sw[k] = 0.f; }
  }
  return mask;
}

}  // namespace

// One CTA of 1024 threads, tokens in chunks of 1024 (one per thread).
// Pass 1 counts the assignments of every local expert with warp ballots (no
// atomics, so no buffer has to be cleared beforehand). Pass 2 ranks each
// warp's 32 tokens per expert with ballots and the warps with a shuffle
// scan, so each expert segment lists its tokens in increasing token order.
// Segments start on multiples of kSegAlign rows; the padding rows carry
// token -1 and weight 0. Also clears the call's device status word.
__device__ __forceinline__ void permute_body(const PermuteParams& p) {
  __shared__ int s_run[kExpertsLocal];
  __shared__ int s_wcnt[32][kExpertsLocal];  // [warp][expert]
  __shared__ int s_wpre[32][kExpertsLocal];
  __shared__ int s_wtouch[32];               // touched tokens per warp

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  if (tid == 0) *p.status = 0;
  if (tid < 4) p.sched[tid] = 0;

  // ---- pass 1: per-expert counts ------------------------------------------
  int my_count = 0;  // lane e of each warp: this warp's tokens choosing expert e
  for (int base = 0; base < p.num_tokens; base += 1024) {
    int sidx[kTopK];
    float sw[kTopK];
    const uint32_t mask = token_selection(p, base + tid, sidx, sw);
#pragma unroll
    for (int e = 0; e < kExpertsLocal; ++e) {
      const uint32_t bal = __ballot_sync(0xffffffffu, (mask >> e) & 1u);
      if (lane == e) my_count += __popc(bal);
    }
  }
  s_wcnt[warp][lane] = my_count;
  __syncthreads();
  if (warp == 0) {
    int c = 0;
#pragma unroll 8
    for (int w = 0; w < 32; ++w) c += s_wcnt[w][lane];
    const int padded = (c + kSegAlign - 1) / kSegAlign * kSegAlign;
    int incl = padded;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    s_run[lane] = incl - padded;
    p.counts[lane] = c;
    p.seg_off[lane + 1] = incl;
    if (lane == 0) p.seg_off[0] = 0;
  }
  __syncthreads();
  // padding rows: expert e = tid / kSegAlign, slot j = tid % kSegAlign
  if (tid < kExpertsLocal * kSegAlign) {
    const int e = tid / kSegAlign;
    const int j = tid % kSegAlign;
    const int c = p.counts[e];
    const int padded = (c + kSegAlign - 1) / kSegAlign * kSegAlign;
    if (c + j < padded) {
      p.perm_tok[s_run[e] + c + j] = -1;
      p.perm_w[s_run[e] + c + j] = 0.f;
      p.perm_row[s_run[e] + c + j] = -1;
    }
  }

  // ---- pass 2: positions and combine rows ---------------------------------
  const uint32_t lt_mask = (1u << lane) - 1u;
  int trun = 0;   // touched tokens of earlier chunks (the same in every thread)
  for (int base = 0; base < p.num_tokens; base += 1024) {
    const int t = base + tid;
    int sidx[kTopK];
    float sw[kTopK];
    const uint32_t mask = token_selection(p, t, sidx, sw);

    // Rank inside the warp, per expert. Ranks of the set bits of `mask` are
    // packed 5 bits each in increasing expert order.
    uint64_t ranks = 0;
    int nset = 0;
    __syncthreads();  // previous chunk's readers of s_wcnt / s_wpre are done
#pragma unroll
    for (int e = 0; e < kExpertsLocal; ++e) {
      const uint32_t bal = __ballot_sync(0xffffffffu, (mask >> e) & 1u);
      if (lane == e) s_wcnt[warp][e] = __popc(bal);
      if ((mask >> e) & 1u) {
        ranks |= static_cast<uint64_t>(__popc(bal & lt_mask)) << (5 * nset);
        ++nset;
      }
    }
    const uint32_t tbal = __ballot_sync(0xffffffffu, mask != 0u);
    if (lane == 0) s_wtouch[warp] = __popc(tbal);
    __syncthreads();

    // Combine row of this token: touched tokens numbered in token order.
    int slot = -1;
    {
      const int wt = s_wtouch[lane];
      int before = lane < warp ? wt : 0;
      int total = wt;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        before += __shfl_xor_sync(0xffffffffu, before, off);
        total += __shfl_xor_sync(0xffffffffu, total, off);
      }
      if (mask != 0u) slot = trun + before + __popc(tbal & lt_mask);
      if (t < p.num_tokens) p.tok_slot[t] = slot;
      if (slot >= 0) p.slot_tok[slot] = t;
      trun += total;
    }

    // Warp w scans expert w over the 32 warps of the chunk.
    {
      const int e = warp;
      const int c = s_wcnt[lane][e];
      int incl = c;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      const int run = s_run[e];
      s_wpre[lane][e] = run + incl - c;
      __syncwarp();
      if (lane == 31) s_run[e] = run + incl;
    }
    __syncthreads();

    uint32_t m = mask;
    int j = 0;
    while (m) {
      const int e = __ffs(m) - 1;
      m &= m - 1;
      const int r = static_cast<int>((ranks >> (5 * j)) & 31u);
      ++j;
      float w = 0.f;
#pragma unroll
      for (int k = 0; k < kTopK; ++k) {
        if (sidx[k] == e) w = sw[k];
      }
      const int pos = s_wpre[warp][e] + r;
      p.perm_tok[pos] = t;
      p.perm_w[pos] = w;
      p.perm_row[pos] = slot;
    }
  }
  if (tid == 0) *p.n_touched = trun;
}

__global__ void __launch_bounds__(1024) permute_kernel(PermuteParams p) {
  pdl_launch_next();
  pdl_wait();
  permute_body(p);
}

namespace {

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA of the cluster arrives; memory operations before
// the barrier (shared::cluster and global) are visible to all CTAs after it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 32-bit store into the shared memory of CTA `rank` of this cluster, at the
// offset `local` has in the calling CTA.
__device__ __forceinline__ void st_cluster_u32(const void* local, uint32_t rank, uint32_t v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(remote), "r"(v) : "memory");
}

}  // namespace

// Decode batches (T <= kDecodeMaxTokens = 64): routing, permutation, the
// permuted row copy and the clears the decode GEMMs rely on, in one cluster
// of 8 CTAs x 256 threads with a single cluster barrier.
//   1. warp w of CTA r routes token 8r + w and stores its eight selections
//      into the shared memory of every CTA of the cluster (distributed
//      shared memory), then starts pulling the token's row into L2 if it
//      has a local pick;
//   2. every CTA derives the whole permutation from its own copy of the
//      selections (warp ballots over 64 tokens: deterministic, segments in
//      increasing token order, padded to kSegAlign rows, the same result as
//      permute_kernel) and writes its share of the permuted index arrays;
//   3. the valid (token, expert) rows are spread over the cluster's 64
//      warps: each copies its rows of the hidden states and their block
//      scales into a_perm / sa_perm and clears the matching g1_acc rows.
// Routing runs on eight SMs rather than one: a warp issues about a thousand
// instructions per token, which on a single SM would serialise 64 tokens.
constexpr int kDecodeMaxRows = kDecodeMaxTokens * kTopK + kExpertsLocal * (kSegAlign - 1);
template <bool kBf16>
__global__ void __cluster_dims__(kDecodeClusterCtas, 1, 1) __launch_bounds__(256)
    route_permute_decode_kernel(RouteParams rp, DecodeFrontParams dp) {
  __shared__ int s_idx[kDecodeMaxTokens * kTopK];   // every CTA holds all selections
  __shared__ float s_w[kDecodeMaxTokens * kTopK];
  __shared__ int s_ptok[kDecodeMaxRows];             // the permutation, per CTA
  __shared__ float s_pw[kDecodeMaxRows];
  __shared__ int s_wcnt[2][kExpertsLocal];
  __shared__ int s_start[kExpertsLocal];
  __shared__ int s_cnt[kExpertsLocal];
  __shared__ int s_cpre[kExpertsLocal];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int T = rp.num_tokens;
  const uint32_t rank = cluster_rank();

  // ---- 1. routing -----------------------------------------------------------
  {
    const int t = static_cast<int>(rank) * 8 + warp;
    if (t < T) {
      int idx;
      float w;
      route_token_any(rp, t, lane, idx, w);
      if (lane < kTopK) {
#pragma unroll
        for (uint32_t q = 0; q < kDecodeClusterCtas; ++q) {
          st_cluster_u32(&s_idx[t * kTopK + lane], q, static_cast<uint32_t>(idx));
          st_cluster_u32(&s_w[t * kTopK + lane], q, __float_as_uint(w));
        }
      }
      // A token with a local pick has its row copied in step 3: start
      // pulling its 7 KB row and 56 block scales into L2 now.
      const int le = idx - dp.local_expert_offset;
      if constexpr (kBf16) {
        if (__ballot_sync(0xffffffffu, lane < kTopK && le >= 0 && le < kExpertsLocal)) {
          const uint8_t* row = reinterpret_cast<const uint8_t*>(dp.hidden_bf16 + static_cast<int64_t>(t) * kHidden);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if ((lane + 32 * k) * 128 < kHidden * 2) prefetch_l2(row + (lane + 32 * k) * 128);
        }
      } else if (__ballot_sync(0xffffffffu, lane < kTopK && le >= 0 && le < kExpertsLocal)) {
        const uint8_t* row = dp.hidden + static_cast<int64_t>(t) * kHidden;
        prefetch_l2(row + lane * 128);
        prefetch_l2(row + (lane + 32) * 128);
        prefetch_l2(dp.hidden_scale + static_cast<int64_t>(lane) * T + t);
        if (lane + 32 < kHiddenBlocks) prefetch_l2(dp.hidden_scale + static_cast<int64_t>(lane + 32) * T + t);
      }
    }
  }
  cluster_sync_all();

  // ---- 2. permutation (every CTA, from its own copy) ------------------------
  {
    const int t = tid;   // token of this thread (warps 0 and 1)
    int sidx[kTopK];
    float sw[kTopK];
    uint32_t mask = 0;
    uint64_t ranks = 0;
    if (warp < 2) {
#pragma unroll
      for (int k = 0; k < kTopK; ++k) {
        sidx[k] = -1;
        sw[k] = 0.f;
        if (t < T) {
          const int le = s_idx[t * kTopK + k] - dp.local_expert_offset;
          if (le >= 0 && le < kExpertsLocal) {
            sidx[k] = le;
            sw[k] = s_w[t * kTopK + k];
            mask |= 1u << le;
          }
        }
      }
      const uint32_t lt_mask = (1u << lane) - 1u;
      int nset = 0;
#pragma unroll
      for (int e = 0; e < kExpertsLocal; ++e) {
        const uint32_t bal = __ballot_sync(0xffffffffu, (mask >> e) & 1u);
        if (lane == e) s_wcnt[warp][e] = __popc(bal);
        if ((mask >> e) & 1u) {
          ranks |= static_cast<uint64_t>(__popc(bal & lt_mask)) << (5 * nset);
          ++nset;
        }
      }
    }
    __syncthreads();
    if (warp == 0) {
      const int c = s_wcnt[0][lane] + s_wcnt[1][lane];
      const int padded = (c + kSegAlign - 1) / kSegAlign * kSegAlign;
      int incl = padded;
      int cincl = c;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, incl, off);
        const int co = __shfl_up_sync(0xffffffffu, cincl, off);
        if (lane >= off) {
          incl += o;
          cincl += co;
        }
      }
      s_start[lane] = incl - padded;
      s_cnt[lane] = c;
      s_cpre[lane] = cincl - c;
      if (rank == 0) {
        dp.counts[lane] = c;
        dp.seg_off[lane + 1] = incl;
        if (lane == 0) dp.seg_off[0] = 0;
        __threadfence();
      }
    } else if (rank == 1 && warp == 2) {
      if (lane < 4) dp.sched[lane] = 0;
      if (lane == 4) *dp.status = 0;
      __threadfence();
    }
    __syncthreads();
    // GEMM1 may start now: the segment table, the cleared unit counter and
    // status word are visible device-wide (fenced above), and GEMM1 reads
    // them and issues its first weight tiles before it waits for this grid
    // to complete (the permuted rows, scales and g1_acc clears below).
    pdl_launch_next();
    if (warp < 2) {
      if (t < T) {
        uint32_t m = mask;
        int j = 0;
        while (m) {
          const int e = __ffs(m) - 1;
          m &= m - 1;
          const int r = static_cast<int>((ranks >> (5 * j)) & 31u) + (warp == 1 ? s_wcnt[0][e] : 0);
          ++j;
          float w = 0.f;
#pragma unroll
          for (int k = 0; k < kTopK; ++k) {
            if (sidx[k] == e) w = sw[k];
          }
          s_ptok[s_start[e] + r] = t;
          s_pw[s_start[e] + r] = w;
        }
      }
    } else {
      // padding rows: 32 experts x kSegAlign slots over threads 64..255
      for (int i = tid - 64; i < kExpertsLocal * kSegAlign; i += blockDim.x - 64) {
        const int e = i / kSegAlign;
        const int j = i % kSegAlign;
        const int c = s_cnt[e];
        const int padded = (c + kSegAlign - 1) / kSegAlign * kSegAlign;
        if (c + j < padded) {
          s_ptok[s_start[e] + c + j] = -1;
          s_pw[s_start[e] + c + j] = 0.f;
        }
      }
    }
    __syncthreads();
    // this CTA's share of the permuted index arrays
    const int nrows = s_start[kExpertsLocal - 1] + (s_cnt[kExpertsLocal - 1] + kSegAlign - 1) / kSegAlign * kSegAlign;
    for (int i = static_cast<int>(rank) * blockDim.x + tid; i < nrows; i += kDecodeClusterCtas * blockDim.x) {
      dp.perm_tok[i] = s_ptok[i];
      dp.perm_w[i] = s_pw[i];
    }
  }

  // ---- 3. permuted rows and g1_acc clears of the valid pairs ---------------
  // Valid pair v (0 <= v < sum of counts) is row s_start[e] + v - s_cpre[e]
  // of expert e. One warp per row.
  {
    const int incl = s_cpre[lane] + s_cnt[lane];
    const int pairs = __shfl_sync(0xffffffffu, incl, 31);
    for (int v = static_cast<int>(rank) * 8 + warp; v < pairs; v += kDecodeClusterCtas * 8) {
      const int e = __popc(__ballot_sync(0xffffffffu, incl <= v));
      const int row = s_start[e] + v - s_cpre[e];
      const int tok = s_ptok[row];
      if constexpr (kBf16) {
        float4* g = reinterpret_cast<float4*>(dp.g1_acc + static_cast<int64_t>(row) * kGemm1Out);
#pragma unroll 8
        for (int i = lane; i < kGemm1Out / 4; i += 32) g[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        quantize_row_1x128(dp.hidden_bf16 + static_cast<int64_t>(tok) * kHidden,
                           dp.a_perm + static_cast<int64_t>(row) * kHidden, lane,
                           [&](int kb, float sc) { dp.sa_perm[static_cast<int64_t>(kb) * dp.cap + row] = sc; });
        continue;
      }
      // every load first, then the stores (the clears do not wait for them)
      const uint4* src = reinterpret_cast<const uint4*>(dp.hidden + static_cast<int64_t>(tok) * kHidden);
      uint4 rowv[kHidden / 16 / 32];
#pragma unroll
      for (int i = 0; i < kHidden / 16 / 32; ++i) rowv[i] = src[lane + 32 * i];
      const float sc0 = dp.hidden_scale[static_cast<int64_t>(lane) * T + tok];
      const float sc1 = lane + 32 < kHiddenBlocks ? dp.hidden_scale[static_cast<int64_t>(lane + 32) * T + tok] : 0.f;
      float4* g = reinterpret_cast<float4*>(dp.g1_acc + static_cast<int64_t>(row) * kGemm1Out);
#pragma unroll 8
      for (int i = lane; i < kGemm1Out / 4; i += 32) g[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      uint4* dst = reinterpret_cast<uint4*>(dp.a_perm + static_cast<int64_t>(row) * kHidden);
#pragma unroll
      for (int i = 0; i < kHidden / 16 / 32; ++i) dst[lane + 32 * i] = rowv[i];
      dp.sa_perm[static_cast<int64_t>(lane) * dp.cap + row] = sc0;
      if (lane + 32 < kHiddenBlocks) dp.sa_perm[static_cast<int64_t>(lane + 32) * dp.cap + row] = sc1;
    }
  }
}

// Multi-CTA permutation for batches of more than 1024 tokens, one chunk of
// kPermChunk tokens (one per thread) per CTA, same result as permute_kernel.
// permute_count_kernel writes each chunk's per-expert counts;
// permute_place_kernel derives the segment starts from all chunks' counts
// and places its chunk's tokens after those of earlier chunks.
constexpr int kChunkStride = kExpertsLocal + 1;   // chunk_counts row: 32 expert counts + touched tokens
constexpr int kPermWarps = kPermChunk / 32;

__global__ void __launch_bounds__(kPermChunk) permute_count_kernel(PermuteParams p) {
  __shared__ int s_wcnt[kPermWarps][kExpertsLocal];
  __shared__ int s_wtouch[kPermWarps];
  pdl_launch_next();
  pdl_wait();
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  int sidx[kTopK];
  float sw[kTopK];
  const uint32_t mask = token_selection(p, blockIdx.x * kPermChunk + tid, sidx, sw);
  int my_count = 0;
#pragma unroll
  for (int e = 0; e < kExpertsLocal; ++e) {
    const uint32_t bal = __ballot_sync(0xffffffffu, (mask >> e) & 1u);
    if (lane == e) my_count = __popc(bal);
  }
  s_wcnt[warp][lane] = my_count;
  const uint32_t tbal = __ballot_sync(0xffffffffu, mask != 0u);
  if (lane == 0) s_wtouch[warp] = __popc(tbal);
  __syncthreads();
  if (warp == 0) {
    int c = 0;
#pragma unroll
    for (int w = 0; w < kPermWarps; ++w) c += s_wcnt[w][lane];
    p.chunk_counts[blockIdx.x * kChunkStride + lane] = c;
    int tt = lane < kPermWarps ? s_wtouch[lane] : 0;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) tt += __shfl_xor_sync(0xffffffffu, tt, off);
    if (lane == 0) p.chunk_counts[blockIdx.x * kChunkStride + kExpertsLocal] = tt;
  }
}

__global__ void __launch_bounds__(kPermChunk) permute_place_kernel(PermuteParams p) {
  __shared__ int s_start[kExpertsLocal];
  __shared__ int s_total[kExpertsLocal];
  __shared__ int s_base[kExpertsLocal];
  __shared__ int s_wcnt[kPermWarps][kExpertsLocal];
  __shared__ int s_wpre[kPermWarps][kExpertsLocal];
  __shared__ int s_wtouch[kPermWarps];
  __shared__ int s_tbase;
  pdl_launch_next();
  pdl_wait();
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int chunk = blockIdx.x;
  if (warp == 1) {
    // touched tokens of earlier chunks (and in all chunks)
    int tb = 0, tt = 0;
    for (int c = lane; c < static_cast<int>(gridDim.x); c += 32) {
      const int v = p.chunk_counts[c * kChunkStride + kExpertsLocal];
      tt += v;
      if (c < chunk) tb += v;
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      tb += __shfl_xor_sync(0xffffffffu, tb, off);
      tt += __shfl_xor_sync(0xffffffffu, tt, off);
    }
    if (lane == 0) {
      s_tbase = tb;
      if (chunk == 0) *p.n_touched = tt;
    }
  }
  {
    // per-expert totals over all chunks and over earlier chunks, each warp
    // taking every kPermWarps-th chunk
    int total = 0, before = 0;
#pragma unroll 4
    for (int c = warp; c < static_cast<int>(gridDim.x); c += kPermWarps) {
      const int v = p.chunk_counts[c * kChunkStride + lane];
      total += v;
      if (c < chunk) before += v;
    }
    s_wcnt[warp][lane] = total;
    s_wpre[warp][lane] = before;
  }
  __syncthreads();
  if (warp == 0) {
    int total = 0, before = 0;
#pragma unroll
    for (int w = 0; w < kPermWarps; ++w) {
      total += s_wcnt[w][lane];
      before += s_wpre[w][lane];
    }
    const int padded = (total + kSegAlign - 1) / kSegAlign * kSegAlign;
    int incl = padded;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    s_start[lane] = incl - padded;
    s_total[lane] = total;
    s_base[lane] = incl - padded + before;
    if (chunk == 0) {
      p.counts[lane] = total;
      p.seg_off[lane + 1] = incl;
      if (lane == 0) {
        p.seg_off[0] = 0;
        *p.status = 0;
      }
      if (lane < 4) p.sched[lane] = 0;
    }
  }
  __syncthreads();
  if (chunk == 0) {
    // padding rows: expert e = i / kSegAlign, slot j = i % kSegAlign
    for (int i = tid; i < kExpertsLocal * kSegAlign; i += kPermChunk) {
      const int e = i / kSegAlign;
      const int j = i % kSegAlign;
      const int c = s_total[e];
      const int padded = (c + kSegAlign - 1) / kSegAlign * kSegAlign;
      if (c + j < padded) {
        p.perm_tok[s_start[e] + c + j] = -1;
        p.perm_w[s_start[e] + c + j] = 0.f;
        p.perm_row[s_start[e] + c + j] = -1;
      }
    }
  }
  const int t = chunk * kPermChunk + tid;
  int sidx[kTopK];
  float sw[kTopK];
  const uint32_t mask = token_selection(p, t, sidx, sw);
  const uint32_t lt_mask = (1u << lane) - 1u;
  uint64_t ranks = 0;
  int nset = 0;
#pragma unroll
  for (int e = 0; e < kExpertsLocal; ++e) {
    const uint32_t bal = __ballot_sync(0xffffffffu, (mask >> e) & 1u);
    if (lane == e) s_wcnt[warp][e] = __popc(bal);
    if ((mask >> e) & 1u) {
      ranks |= static_cast<uint64_t>(__popc(bal & lt_mask)) << (5 * nset);
      ++nset;
    }
  }
  const uint32_t tbal = __ballot_sync(0xffffffffu, mask != 0u);
  if (lane == 0) s_wtouch[warp] = __popc(tbal);
  __syncthreads();
  {
    // first row of this warp's tokens of expert `lane`: after earlier chunks'
    // and this chunk's earlier warps' tokens of that expert
    int before = 0;
    for (int w = 0; w < warp; ++w) before += s_wcnt[w][lane];
    s_wpre[warp][lane] = s_base[lane] + before;
  }
  int slot = -1;
  {
    int before = lane < warp ? s_wtouch[lane] : 0;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) before += __shfl_xor_sync(0xffffffffu, before, off);
    if (mask != 0u) slot = s_tbase + before + __popc(tbal & lt_mask);
    if (t < p.num_tokens) p.tok_slot[t] = slot;
    if (slot >= 0) p.slot_tok[slot] = t;
  }
  __syncthreads();
  uint32_t m = mask;
  int j = 0;
  while (m) {
    const int e = __ffs(m) - 1;
    m &= m - 1;
    const int r = static_cast<int>((ranks >> (5 * j)) & 31u);
    ++j;
    float w = 0.f;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
      if (sidx[k] == e) w = sw[k];
    }
    const int pos = s_wpre[warp][e] + r;
    p.perm_tok[pos] = t;
    p.perm_w[pos] = w;
    p.perm_row[pos] = slot;
  }
}

// Copies every permuted row's activations and block scales into contiguous
// buffers (one warp per row): a_perm[r, :] = hidden[tok(r), :] and
// sa_perm[kb, r] = hidden_scale[kb, tok(r)].
// This replaces per-row TMA gathers inside GEMM1 with plain 2-D tiles.
// It also clears the rows of the combine buffer y_acc that GEMM2 adds into
// (one per token with a local pick).
__global__ void __launch_bounds__(256) gather_rows_kernel(GatherParams p) {
  // Releases GEMM1 only after the permutation has completed: GEMM1 reads the
  // segment table before its own wait to prefetch weight tiles.
  pdl_wait();
  pdl_launch_next();
  const int rows = p.seg_off[kExpertsLocal];
  const int lane = threadIdx.x & 31;
  const int warps_total = gridDim.x * (blockDim.x >> 5);
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t y4 = static_cast<int64_t>(*p.n_touched) * (kHidden / 4);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < y4; i += nthreads)
    reinterpret_cast<float4*>(p.y_acc)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (p.g1_acc != nullptr) {
    // token-major GEMM1 K-split sums start from zero when the split is on
    int units = (p.counts[lane] + 127) / 128 * kInterBlocks;   // lane = expert
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) units += __shfl_xor_sync(0xffffffffu, units, off);
    if (tm_gemm1_splits(units) > 1) {
      const int64_t g4 = static_cast<int64_t>(rows) * (kGemm1Out / 4);
      for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < g4; i += nthreads)
        reinterpret_cast<float4*>(p.g1_acc)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  // Padding rows are skipped: they only ever feed token columns or rows that
  // the GEMM epilogues discard, and every output column depends on its own
  // token row alone.
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps_total) {
    const int tok = p.perm_tok[r];
    if (tok < 0) continue;
    uint4* dst = reinterpret_cast<uint4*>(p.a_perm + static_cast<int64_t>(r) * kHidden);
    const uint4* src = reinterpret_cast<const uint4*>(p.hidden + static_cast<int64_t>(tok) * kHidden);
    // loads first, then stores (two halves of the row): the stores may alias
    // the loads as far as the compiler knows, so interleaving them would keep
    // one load in flight at a time
    constexpr int kHalf = kHidden / 16 / 32 / 2;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint4 v[kHalf];
#pragma unroll
      for (int i = 0; i < kHalf; ++i) v[i] = src[lane + 32 * (h * kHalf + i)];
#pragma unroll
      for (int i = 0; i < kHalf; ++i) dst[lane + 32 * (h * kHalf + i)] = v[i];
    }
    for (int kb = lane; kb < kHiddenBlocks; kb += 32)
      p.sa_perm[static_cast<int64_t>(kb) * p.cap + r] = p.hidden_scale[static_cast<int64_t>(kb) * p.num_tokens + tok];
  }
}

template __global__ void route_permute_decode_kernel<false>(RouteParams, DecodeFrontParams);
template __global__ void route_permute_decode_kernel<true>(RouteParams, DecodeFrontParams);

}  // namespace moe
