// Backward pass of the routed micro-expert layer: the elementwise and
// per-row kernels between the grouped GEMMs (abi.cu spx_layer_backward runs
// the GEMMs on the tcgen05 engine of gemm.cu).
//
// The steps mirror what PyTorch autograd does through the reference forward
// in BF16 (mESmaC/spalmer src/spalmer): every tensor the reference holds in
// BF16 is rounded to BF16 here at the same point, arithmetic in between is
// FP32.  The gradient formulas:
//   experts (experts/bank.py:760-778, bank.py:970-978):
//     sg = bf16(silu(g)), h = bf16(sg * u)                    (forward values)
//     dh = bf16(dh' * w), dh' = bf16(dY_t @ D_e^T)            (dh' from the GEMM)
//     d_sg = bf16(dh * u), d_u = bf16(dh * sg)
//     d_g = bf16(d_sg * sigmoid(g) * (1 + g * (1 - sigmoid(g))))
//     d_w = sum_i dh'_i * h_i      (= sum over d of dY_t * y, y = h @ D_e)
//   selection (experts/router.py:92-94): w = softmax(-s_sel)
//     d_s_sel = -bf16(w * (d_w - sum_j w_j d_w_j))
//   load balance (experts/losses.py:58-70), aux = m * sum_e f_e * mean_t p_te:
//     d_p_te = bf16(bf16(bf16(d_aux * m) * f_e) / T)
//     d_s_te = -bf16(p_te * (d_p_te - sum_e p_te d_p_te)),  p = bf16(softmax(-s))
//   softplus (experts/router.py:56): d_logit = bf16(d_s * sigmoid(logit)),
//     or d_s itself past the threshold 20.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"
#include "sm100.cuh"

namespace spx {

namespace {

__device__ __forceinline__ float bfr(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ uint16_t bfbits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
// Two values rounded to BF16 (nearest even) by one packed conversion: the
// word (lo in the low half) and, widened back in place, the rounded floats.
__device__ __forceinline__ uint32_t bfr2(float& lo, float& hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  const uint32_t w = *reinterpret_cast<uint32_t*>(&v);
  lo = __uint_as_float(w << 16);
  hi = __uint_as_float(w & 0xFFFF0000u);
  return w;
}

int grid_for(int64_t items, int per_block) {
  int64_t g = (items + per_block - 1) / per_block;
  if (g > 148 * 32) g = 148 * 32;
  return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace

// SwiGLU backward.  gu holds the pre-activations in the forward GEMM1's
// chunk layout (chunk n: c gate columns, then c up columns), dhp =
// bf16(dY_t @ D_e^T).  Writes bf16(h * w) (the forward hidden row times the
// routing weight: the down projection's weight gradient is
// sum_p bf16(h_p w_p)^T dU_p; h itself for unit weights), [d_gate | d_up]
// with the up half at column kI (zero padded to 2 kI), and d_w of the pair in
// pair order (order[p]).  A row is handled by `lanes` consecutive threads of a
// warp, 8 hidden columns (16-byte loads and stores) each; needs c % 8 == 0.
__device__ __forceinline__ void swiglu_bwd8(const uint4& gv, const uint4& uv, const uint4& dv, float w,
                                            uint4& hv, uint4& dgv, uint4& duv, float& part) {
  const uint32_t G[4] = {gv.x, gv.y, gv.z, gv.w}, U[4] = {uv.x, uv.y, uv.z, uv.w}, D[4] = {dv.x, dv.y, dv.z, dv.w};
  uint32_t H[4], DG[4], DU[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    // The word's two columns side by side ([0] low half, [1] high half), each
    // rounding done for both at once.
    const float g[2] = {__uint_as_float(G[q] << 16), __uint_as_float(G[q] & 0xFFFF0000u)};
    const float u[2] = {__uint_as_float(U[q] << 16), __uint_as_float(U[q] & 0xFFFF0000u)};
    const float dh1[2] = {__uint_as_float(D[q] << 16), __uint_as_float(D[q] & 0xFFFF0000u)};
    float sgm[2], sg[2], h[2], dh[2], dsg[2], du[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float den = 1.0f + expf(-g[i]);  // one exponential for both (sigmoidf_'s and silu's)
      sgm[i] = 1.0f / den;
      sg[i] = g[i] / den;  // silu as the reference evaluates it
    }
    bfr2(sg[0], sg[1]);
    h[0] = sg[0] * u[0];
    h[1] = sg[1] * u[1];
    bfr2(h[0], h[1]);
    part += dh1[0] * h[0];
    part += dh1[1] * h[1];
    float hw[2] = {h[0] * w, h[1] * w};  // the weighted row for the down projection's weight gradient
    H[q] = bfr2(hw[0], hw[1]);
    dh[0] = dh1[0] * w;
    dh[1] = dh1[1] * w;
    bfr2(dh[0], dh[1]);
    dsg[0] = dh[0] * u[0];
    dsg[1] = dh[1] * u[1];
    bfr2(dsg[0], dsg[1]);
    du[0] = dh[0] * sg[0];
    du[1] = dh[1] * sg[1];
    DU[q] = bfr2(du[0], du[1]);
    float dg0 = dsg[0] * (sgm[0] * (1.0f + g[0] * (1.0f - sgm[0])));
    float dg1 = dsg[1] * (sgm[1] * (1.0f + g[1] * (1.0f - sgm[1])));
    DG[q] = bfr2(dg0, dg1);
  }
  hv = make_uint4(H[0], H[1], H[2], H[3]);
  dgv = make_uint4(DG[0], DG[1], DG[2], DG[3]);
  duv = make_uint4(DU[0], DU[1], DU[2], DU[3]);
}

__global__ void bwd_swiglu_kernel(const uint16_t* __restrict__ gu, int ld_gu, int c, const uint16_t* __restrict__ dhp,
                                  int ld_dhp, const uint16_t* __restrict__ sorted_w, const int* __restrict__ order,
                                  int64_t P, int I, int kI, int lanes, uint16_t* __restrict__ h_sorted,
                                  uint16_t* __restrict__ dgu, float* __restrict__ dw_pair) {
  const int lane = threadIdx.x & 31;
  const int sub = lane % lanes;            // position within the row group
  const int group = lane / lanes;          // row group within the warp
  const int groups = 32 / lanes;
  const unsigned gmask = (lanes == 32) ? 0xFFFFFFFFu : (((1u << lanes) - 1u) << (group * lanes));
  const int64_t nslots = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5) * groups;
  const int64_t slot0 = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * groups + group;
  const int64_t iters = (P + nslots - 1) / nslots;  // uniform over the warp: every lane runs the shuffles
  for (int64_t it = 0; it < iters; ++it) {
    const int64_t p = slot0 + it * nslots;
    const bool live = p < P;
    float part = 0.0f;
    if (live) {
      const float w = bf16_to_f32(sorted_w[p]);
      const uint16_t* grow = gu + p * ld_gu;
      for (int i = 8 * sub; i < 2 * kI; i += 8 * lanes) {
        if (i < I) {
          const int chunk = i / c, j = i - chunk * c;
          const uint4 gv = *reinterpret_cast<const uint4*>(grow + chunk * 2 * c + j);
          const uint4 uv = *reinterpret_cast<const uint4*>(grow + chunk * 2 * c + c + j);
          const uint4 dv = *reinterpret_cast<const uint4*>(dhp + p * ld_dhp + i);
          uint4 hv, dgv, duv;
          swiglu_bwd8(gv, uv, dv, w, hv, dgv, duv, part);
          *reinterpret_cast<uint4*>(h_sorted + p * I + i) = hv;
          *reinterpret_cast<uint4*>(dgu + p * 2 * kI + i) = dgv;
          *reinterpret_cast<uint4*>(dgu + p * 2 * kI + kI + i) = duv;
        } else if (i < kI) {
          // K padding of both halves
          *reinterpret_cast<uint4*>(dgu + p * 2 * kI + i) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(dgu + p * 2 * kI + kI + i) = make_uint4(0, 0, 0, 0);
        }
      }
    }
    for (int off = lanes / 2; off >= 1; off >>= 1) part += __shfl_xor_sync(gmask, part, off);
    if (live && sub == 0) dw_pair[order[p]] = part;
  }
}

// Router backward, one warp per token row: selection softmax, load-balance
// softmax, optional upstream score gradient, softplus.  Lanes own columns
// lane, lane + 32, ...; the row's k selected experts are distinct.
template <int NQ>
__global__ void bwd_router_kernel(const BwdRouterArgs a) {
  const int lane = threadIdx.x & 31;
  const int E = a.num_experts, k = a.top_k;
  // eligible expert count m (resident experts, or E)
  int m = E;
  if (a.resident != nullptr) {
    int cnt = 0;
    for (int c = lane; c < E; c += 32) cnt += a.resident[c] ? 1 : 0;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) cnt += __shfl_xor_sync(0xFFFFFFFFu, cnt, off);
    m = cnt;
  }
  const float g_aux = a.d_aux != nullptr ? bf16_to_f32(*a.d_aux) : 0.0f;
  const float gs = bfr(g_aux * bfr(static_cast<float>(m)));  // d(sum) = d_aux * eligible
  // Per column, the same for every row: eligibility and the load-balance
  // gradient of the mean probability, d_p = bf16(bf16(gs * f_e) / T).
  bool ok[NQ];
  float dp[NQ];
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    const int c = lane + 32 * q;
    ok[q] = c < E && (a.resident == nullptr || a.resident[c] != 0);
    const float f = c < E ? bfr(a.fractions[c]) : 0.0f;
    dp[q] = ok[q] ? bfr(bfr(gs * f) / static_cast<float>(a.tokens)) : 0.0f;
  }
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); t < a.tokens;
       t += nwarps) {
    const uint16_t* srow = a.scores + t * E;
    float s[NQ], acc[NQ];
    float mx = -INFINITY;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      const int c = lane + 32 * q;
      s[q] = c < E ? bf16_to_f32(srow[c]) : 0.0f;
      acc[q] = 0.0f;
      if (ok[q]) mx = fmaxf(mx, -s[q]);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, off));
    // ---- load balance: p = bf16(softmax(-s)), d_p = bf16(bf16(gs * f_e) / T)
    if (a.d_aux != nullptr) {
      float e[NQ], sum = 0.0f;
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        e[q] = ok[q] ? expf(-s[q] - mx) : 0.0f;
        sum += e[q];
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, off);
      float p[NQ], dot = 0.0f;
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        p[q] = ok[q] ? bfr(e[q] / sum) : 0.0f;
        dot += p[q] * dp[q];
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) dot += __shfl_xor_sync(0xFFFFFFFFu, dot, off);
#pragma unroll
      for (int q = 0; q < NQ; ++q)
        if (ok[q]) acc[q] -= bfr(p[q] * (dp[q] - dot));
    }
    // ---- selection softmax: w = softmax(-s_sel), d_w from the experts
    float w = 0.0f, dw = 0.0f;
    int id = -1;
    if (lane < k) {
      id = static_cast<int>(a.ids[t * k + lane]);
      w = bf16_to_f32(a.weights[t * k + lane]);
      dw = bfr(a.dw[t * k + lane]);
    }
    float wdw = w * dw;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) wdw += __shfl_xor_sync(0xFFFFFFFFu, wdw, off);
    const float dsel = lane < k ? -bfr(w * (dw - wdw)) : 0.0f;
    for (int j = 0; j < k; ++j) {
      const int cj = __shfl_sync(0xFFFFFFFFu, id, j);
      const float vj = __shfl_sync(0xFFFFFFFFu, dsel, j);
#pragma unroll
      for (int q = 0; q < NQ; ++q)
        if (lane + 32 * q == cj) acc[q] += vj;
    }
    // ---- upstream score gradient, softplus, store
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      const int c = lane + 32 * q;
      if (c < E) {
        float ds = acc[q];
        if (a.d_scores != nullptr) ds += bf16_to_f32(a.d_scores[t * E + c]);
        ds = bfr(ds);
        float dl = ds;
        if (a.logits != nullptr) {
          const float x = bf16_to_f32(a.logits[t * E + c]);
          if (!(x > 20.0f)) dl = ds * sigmoidf_(x);
        }
        a.d_logits[t * E + c] = bfbits(dl);
      }
    }
  }
}

int launch_bwd_swiglu(const uint16_t* gu, int ld_gu, int c, const uint16_t* dhp, int ld_dhp,
                      const uint16_t* sorted_w, const int* order, int64_t P, int I, int kI, uint16_t* h_sorted,
                      uint16_t* dgu, float* dw_pair, cudaStream_t stream) {
  if (c % 8 != 0 || I % 8 != 0 || ld_gu % 8 != 0 || ld_dhp % 8 != 0) return SPX_ERR_UNSUPPORTED;
  int lanes = 1;  // threads per row: enough for 8 columns each, a power of two <= 32
  while (lanes < 32 && 8 * lanes < kI) lanes <<= 1;
  const int rows_per_block = 8 * (32 / lanes);
  bwd_swiglu_kernel<<<grid_for(P, rows_per_block), 256, 0, stream>>>(gu, ld_gu, c, dhp, ld_dhp, sorted_w, order, P,
                                                                     I, kI, lanes, h_sorted, dgu, dw_pair);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

int launch_bwd_router(const BwdRouterArgs& a, cudaStream_t stream) {
  if (a.tokens <= 0) return SPX_OK;
  if (a.top_k > 32 || a.num_experts > 1024) return SPX_ERR_UNSUPPORTED;
  const int grid = grid_for(a.tokens, 8);
  const int nq = (a.num_experts + 31) / 32;
  if (nq <= 8)
    bwd_router_kernel<8><<<grid, 256, 0, stream>>>(a);
  else
    bwd_router_kernel<32><<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? SPX_OK : SPX_ERR_CUDA;
}

}  // namespace spx
