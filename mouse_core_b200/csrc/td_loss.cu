// K12: the one-step TD loss of DqnObjective, its metrics and its gradient.
//
// Replaces DqnObjective.__call__ (src/mouse_core/objectives/dqn.py:116-213)
// and _valid_transitions (dqn.py:12-39) on the device: pair (i, i + 1) is a
// transition iff both steps share a sequence id; the fields stored at i + 1
// (action, reward, done code) describe the transition out of step i; the
// target is reward + gamma[done] * max_a q_target[i + 1]; the loss is the mean
// over valid pairs of (q[i, a] - target)^2 (+ cql_weight * (|target| + eps) *
// (logsumexp(q[i]) - q[i, a]) when CQL is on). The reference builds ~15 small
// tensors for this and reads its metrics back with a host sync; here one
// kernel computes every pair's error and per-block partial sums, and the last
// block to finish reduces the partials in a fixed order (so the result does
// not depend on scheduling) into loss and metrics: mean / std / min / max over
// valid pairs of max_a q[i] — no host sync. A second kernel writes the
// gradient d loss / d q from the saved per-pair errors.
#include "common.cuh"
#include "kernels.h"

namespace mb {

constexpr int kTdThreads = 256;
constexpr int kTdStats = 6;  // loss sum, valid count, sum, sum of squares, min, max of max_a q

__global__ void __launch_bounds__(kTdThreads) td_loss_fwd_kernel(TdParams p) {
  __shared__ float red[kTdStats][kTdThreads / 32];
  __shared__ int last;
  float ls = 0.f, cnt = 0.f, s1 = 0.f, s2 = 0.f, mn = INFINITY, mx = -INFINITY;
  const int pairs = p.N - 1;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < pairs; i += gridDim.x * blockDim.x) {
    const bool valid = p.seq == nullptr || p.seq[i + 1] == p.seq[i];
    const long long a = p.action[i + 1];
    const long long d = p.done[i + 1];
    float err = 0.f, cql = 0.f, qmax = -INFINITY;
    bool ok = false;
    if (valid) {
      if (a < 0 || a >= p.A || d < 0 || d > 4) {
        report(kDevBadIndex);  // the reference's indexing would raise; the pair is left out
      } else {
        ok = true;
        const float* qi = p.q + (size_t)i * p.A;
        const float* qt = p.q_target + (size_t)(i + 1) * p.A;
        float tmax = -INFINITY;
        for (int k = 0; k < p.A; ++k) {
          tmax = fmaxf(tmax, qt[k]);
          qmax = fmaxf(qmax, qi[k]);
        }
        const float target = p.reward[i + 1] + p.gamma[d] * tmax;
        err = qi[a] - target;
        float l = err * err;
        if (p.cql_weight > 0.f) {
          float se = 0.f;
          for (int k = 0; k < p.A; ++k) se += expf(qi[k] - qmax);
          cql = qmax + logf(se) - qi[a];  // logsumexp(q_i) - q_i[a]
          l += p.cql_weight * (fabsf(target) + p.cql_eps) * cql;
          p.cql_scale[i] = fabsf(target) + p.cql_eps;
        }
        ls += l;
        cnt += 1.f;
        s1 += qmax;
        s2 += qmax * qmax;
        mn = fminf(mn, qmax);
        mx = fmaxf(mx, qmax);
      }
    }
    p.err[i] = ok ? err : 0.f;
    p.valid[i] = ok ? 1 : 0;
  }
  // Block reduction (fixed order), partials to scratch.
  float v[kTdStats] = {ls, cnt, s1, s2, mn, mx};
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int k = 0; k < kTdStats; ++k) {
    float x = v[k];
    for (int o = 16; o > 0; o >>= 1) {
      const float y = __shfl_xor_sync(0xffffffffu, x, o);
      x = k == 4 ? fminf(x, y) : (k == 5 ? fmaxf(x, y) : x + y);
    }
    if (lane == 0) red[k][w] = x;
  }
  __syncthreads();
  if (threadIdx.x < kTdStats) {
    const int k = threadIdx.x;
    float x = red[k][0];
    for (int j = 1; j < kTdThreads / 32; ++j) x = k == 4 ? fminf(x, red[k][j]) : (k == 5 ? fmaxf(x, red[k][j]) : x + red[k][j]);
    p.partials[blockIdx.x * kTdStats + k] = x;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(p.ticket, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  if (threadIdx.x == 0) {
    __threadfence();
    double t[kTdStats] = {0, 0, 0, 0, INFINITY, -INFINITY};
    for (int b = 0; b < (int)gridDim.x; ++b) {
      const float* pb = p.partials + b * kTdStats;
      t[0] += __ldcg(pb + 0);
      t[1] += __ldcg(pb + 1);
      t[2] += __ldcg(pb + 2);
      t[3] += __ldcg(pb + 3);
      t[4] = fmin(t[4], (double)__ldcg(pb + 4));
      t[5] = fmax(t[5], (double)__ldcg(pb + 5));
    }
    const double n = t[1];
    const double mean = t[2] / n;
    const double var = n > 1 ? (t[3] - n * mean * mean) / (n - 1) : 0.0;  // unbiased, as torch.std
    p.out[0] = (float)(t[0] / n);  // loss (NaN when no pair is valid)
    p.out[1] = (float)n;           // valid pairs
    p.out[2] = (float)mean;        // q_values_mean
    p.out[3] = (float)sqrt(var > 0 ? var : 0.0);  // q_values_std
    p.out[4] = (float)t[4];        // q_values_min
    p.out[5] = (float)t[5];        // q_values_max
    *p.ticket = 0;                 // ready for the next call
  }
}

// dq = d loss / d q: 2 err_i / n at [i, a_{i+1}] for valid pairs (+ the CQL
// term's gradient), zero elsewhere (every row, the last one included).
__global__ void __launch_bounds__(kTdThreads) td_loss_bwd_kernel(TdParams p, const float* grad_out) {
  const float n = p.out[1];
  const float g = grad_out ? grad_out[0] : 1.f;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.N; i += gridDim.x * blockDim.x) {
    float* dq = p.dq + (size_t)i * p.A;
    for (int k = 0; k < p.A; ++k) dq[k] = 0.f;
    if (i >= p.N - 1 || !p.valid[i] || !(n > 0.f)) continue;
    const int a = (int)p.action[i + 1];
    dq[a] = 2.f * p.err[i] * g / n;
    if (p.cql_weight > 0.f) {
      const float* qi = p.q + (size_t)i * p.A;
      float qmax = -INFINITY;
      for (int k = 0; k < p.A; ++k) qmax = fmaxf(qmax, qi[k]);
      float se = 0.f;
      for (int k = 0; k < p.A; ++k) se += expf(qi[k] - qmax);
      const float c = p.cql_weight * p.cql_scale[i] * g / n;
      for (int k = 0; k < p.A; ++k) dq[k] += c * (expf(qi[k] - qmax) / se - (k == a ? 1.f : 0.f));
    }
  }
}

int td_blocks(int N) {
  return std::max(1, std::min((N + kTdThreads - 1) / kTdThreads, 148 * 4));
}

cudaError_t launch_td_loss_fwd(const TdParams& p, cudaStream_t stream) {
  td_loss_fwd_kernel<<<td_blocks(p.N), kTdThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_td_loss_bwd(const TdParams& p, const float* grad_out, cudaStream_t stream) {
  td_loss_bwd_kernel<<<td_blocks(p.N), kTdThreads, 0, stream>>>(p, grad_out);
  return cudaGetLastError();
}

}  // namespace mb
