// Gated DeltaNet kernels: the recurrent scan (deltanet_recur.wgsl) with optional fused g/beta
// prologue (deltanet_gbeta.wgsl) and gated-RMSNorm epilogue (deltanet_norm_gate.wgsl), plus the
// stand-alone elementwise kernels and the attention output gate (gate_sigmoid.wgsl).
//
// Recurrence layout: the per-head state S[dk][dv] splits by value column -- every column evolves
// independently (kv = Kn.S[:,dv], delta[dv], S[:,dv] += Kn*delta[dv]) -- so a CTA owns 32
// columns of one head and a head spreads over DV/32 CTAs (4 for DV=128: 192 CTAs for the 27B's
// 48 value heads instead of 48).  Within a CTA, warp w holds rows [w*DK/4, (w+1)*DK/4) of the 32
// columns in registers (lane = column), so the state streams HBM -> registers -> HBM once per
// launch.  The two reductions over dk per token (kv and the output) cross the 4 warps through
// shared memory.  With the fused norm-gate the DV/32 CTAs of a head form a thread-block cluster
// and add their per-token sums of squares through distributed shared memory.
#include <cooperative_groups.h>
#include <math.h>
#include <stdlib.h>

#include "kv.h"
#include "tma.cuh"

namespace cg = cooperative_groups;

namespace bg {
namespace {

__device__ __forceinline__ float softplus_stable(float x) { return fmaxf(x, 0.f) + logf(1.0f + expf(-fabsf(x))); }
__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

template <int DK, bool FUSED>
__global__ void __launch_bounds__(128) deltanet_kernel(DeltaArgs a) {
  constexpr int RPW = DK / 4;      // state rows per warp
  constexpr int KPL = DK / 32;     // k/q values per lane for the norms
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t cg_idx = blockIdx.x;          // column group
  const uint32_t h = blockIdx.y;
  const uint32_t hk = h % a.HK;                // "tile" GQA (deltanet_recur.wgsl:27)
  const uint32_t c = cg_idx * 32 + lane;       // value column
  const bool cval = c < a.DV;

  __shared__ float kn_s[4][DK], qn_s[4][DK];   // per-warp copies (no block barrier needed)
  __shared__ float red_kv[4][32], red_o[4][32];
  __shared__ float ss_part[2];                 // fused: this CTA's sum of squares, double-buffered

  float s[RPW];
  const uint64_t sbase = (uint64_t)h * DK * a.DV;
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const uint32_t dk = warp * RPW + i;
    s[i] = (a.loadState && a.state_in && cval) ? a.state_in[sbase + (uint64_t)dk * a.DV + c] : 0.f;
  }
  const float qscale = 1.0f / sqrtf((float)DK);

  for (uint32_t t = 0; t < a.S; ++t) {
    const uint32_t tt = t + a.tOff;
    const uint64_t base = (uint64_t)tt * a.H + h;
    const uint64_t basek = (uint64_t)tt * a.HK + hk;
    // l2norm(k), l2norm(q)/sqrt(dk): each warp computes both norms on its own (no barrier)
    float kv_[KPL], qv_[KPL];
#pragma unroll
    for (int i = 0; i < KPL; ++i) {
      kv_[i] = a.k[basek * DK + lane * KPL + i];
      qv_[i] = a.q[basek * DK + lane * KPL + i];
    }
    float sk = 0.f, sq = 0.f;
#pragma unroll
    for (int i = 0; i < KPL; ++i) {
      sk = fmaf(kv_[i], kv_[i], sk);
      sq = fmaf(qv_[i], qv_[i], sq);
    }
    sk = warp_sum(sk);
    sq = warp_sum(sq);
    const float ik = 1.0f / sqrtf(sk + 1e-6f);
    const float iq = (1.0f / sqrtf(sq + 1e-6f)) * qscale;
#pragma unroll
    for (int i = 0; i < KPL; ++i) {
      kn_s[warp][lane * KPL + i] = kv_[i] * ik;
      qn_s[warp][lane * KPL + i] = qv_[i] * iq;
    }
    float gt, bt;
    if constexpr (FUSED) {
      const float x = a.a[base] + a.dt_bias[h];
      gt = expf(a.a_neg[h] * softplus_stable(x));
      bt = sigmoidf_(a.b[base]);
    } else {
      gt = expf(a.g[base]);
      bt = a.beta[a.betaOff + base];
    }
    __syncwarp();
    float part = 0.f;
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      s[i] *= gt;
      part = fmaf(s[i], kn_s[warp][warp * RPW + i], part);
    }
    red_kv[warp][lane] = part;
    __syncthreads();
    const float kvv = red_kv[0][lane] + red_kv[1][lane] + red_kv[2][lane] + red_kv[3][lane];
    const float vv = cval ? a.v[base * a.DV + c] : 0.f;
    const float delta = (vv - kvv) * bt;
    float po = 0.f;
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      s[i] = fmaf(kn_s[warp][warp * RPW + i], delta, s[i]);
      po = fmaf(s[i], qn_s[warp][warp * RPW + i], po);
    }
    red_o[warp][lane] = po;
    __syncthreads();
    const float o = red_o[0][lane] + red_o[1][lane] + red_o[2][lane] + red_o[3][lane];
    if (warp == 0 && cval && a.core) a.core[base * a.DV + c] = o;
    if constexpr (FUSED) {
      cg::cluster_group cl = cg::this_cluster();
      if (warp == 0) {
        const float sq2 = warp_sum(cval ? o * o : 0.f);
        if (lane == 0) ss_part[t & 1] = sq2;
      }
      cl.sync();
      if (warp == 0) {
        float tot = 0.f;
        const unsigned nr = cl.num_blocks();
        for (unsigned r = 0; r < nr; ++r) tot += cl.map_shared_rank(&ss_part[t & 1], r)[0];
        const float inv = 1.0f / sqrtf(tot / (float)a.DV + a.eps);
        if (cval) {
          const float zz = a.z[base * a.DV + c];
          a.y[base * a.DV + c] = a.gamma[c] * (o * inv) * (zz / (1.0f + expf(-zz)));
        }
      }
    }
  }
  if constexpr (FUSED) cg::this_cluster().sync();  // no CTA exits while a peer may read its smem
  if (cval && a.state_out) {
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const uint32_t dk = warp * RPW + i;
      a.state_out[sbase + (uint64_t)dk * a.DV + c] = s[i];
    }
  }
}

// Head-per-CTA recurrence for DK = DV = 128 (the 27B's linear layers): 512 threads, warp w owns
// state rows [32*(w/4), 32*(w/4)+32) of columns [32*(w%4), +32) in registers (lane = column).
// Every reduction of a token stays inside the CTA -- kv and the output over dk through shared
// memory, the gated norm's sum of squares over dv with a block reduction -- so no cluster barrier
// is needed, and the next token's inputs are loaded while the current token is processed.  The
// gated norm of token t is finished behind token t+1's first barrier (three barriers per token).
template <bool FUSED>
__global__ void __launch_bounds__(512) deltanet_head_kernel(DeltaArgs a) {
  constexpr int DK = 128, DV = 128, RPW = 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cgp = warp & 3, rq = warp >> 2;
  const uint32_t h = blockIdx.x, hk = h % a.HK;
  const uint32_t c = cgp * 32 + lane;
  __shared__ float kn_s[DK], qn_s[DK];
  __shared__ float red_kv[4][DV], red_o[4][DV];
  __shared__ float ss_s[4];

  // inputs of token t: warp 0 / 1 carry four k / q values per lane, every thread v[c], the
  // norm's z[c] (row-quarter-0 warps) and the per-head gate scalars
  float kq[4], vv, zz = 0.f, ga, gb;
  auto load_inputs = [&](uint32_t t) {
    const uint32_t tt = t + a.tOff;
    const uint64_t base = (uint64_t)tt * a.H + h, basek = (uint64_t)tt * a.HK + hk;
    if (warp < 2) {
      const float4 x = *reinterpret_cast<const float4 *>((warp ? a.q : a.k) + basek * DK + lane * 4);
      kq[0] = x.x; kq[1] = x.y; kq[2] = x.z; kq[3] = x.w;
    }
    vv = a.v[base * DV + c];
    if constexpr (FUSED) {
      if (rq == 0) zz = a.z[base * DV + c];
      ga = a.a[base];
      gb = a.b[base];
    } else {
      ga = a.g[base];
      gb = a.beta[a.betaOff + base];
    }
  };
  if (a.S) load_inputs(0);  // in flight together with the state loads

  float s[RPW];
  const uint64_t sbase = (uint64_t)h * DK * DV;
#pragma unroll
  for (int i = 0; i < RPW; ++i)
    s[i] = (a.loadState && a.state_in) ? a.state_in[sbase + (uint64_t)(rq * RPW + i) * DV + c] : 0.f;
  const float qscale = 1.0f / sqrtf((float)DK);
  const float an = FUSED ? a.a_neg[h] : 0.f, dtb = FUSED ? a.dt_bias[h] : 0.f;
  const float gam = (FUSED && rq == 0) ? a.gamma[c] : 0.f;
  float o_prev = 0.f, z_prev = 0.f;
  uint64_t out_prev = 0;

  for (uint32_t t = 0; t < a.S; ++t) {
    const uint64_t base = (uint64_t)(t + a.tOff) * a.H + h;
    // ---- A: l2norm(k), l2norm(q)/sqrt(dk); g, beta ----
    if (warp < 2) {
      float ss = kq[0] * kq[0] + kq[1] * kq[1] + kq[2] * kq[2] + kq[3] * kq[3];
      ss = warp_sum(ss);
      const float inv = (1.0f / sqrtf(ss + 1e-6f)) * (warp ? qscale : 1.0f);
      float *dst = (warp ? qn_s : kn_s) + lane * 4;
      dst[0] = kq[0] * inv; dst[1] = kq[1] * inv; dst[2] = kq[2] * inv; dst[3] = kq[3] * inv;
    }
    float gt, bt;
    if constexpr (FUSED) {
      gt = expf(an * softplus_stable(ga + dtb));
      bt = sigmoidf_(gb);
    } else {
      gt = expf(ga);
      bt = gb;
    }
    const float v_t = vv, z_t = zz;
    if (t + 1 < a.S) load_inputs(t + 1);
    __syncthreads();
    // the previous token's gated norm: its sum of squares is complete behind this barrier
    if (FUSED && rq == 0 && t > 0) {
      const float inv = 1.0f / sqrtf((ss_s[0] + ss_s[1] + ss_s[2] + ss_s[3]) / (float)DV + a.eps);
      a.y[out_prev] = gam * (o_prev * inv) * (z_prev / (1.0f + expf(-z_prev)));
    }
    // ---- B: decay, kv = Kn . S ----
    float part = 0.f;
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      s[i] *= gt;
      part = fmaf(s[i], kn_s[rq * RPW + i], part);
    }
    red_kv[rq][c] = part;
    __syncthreads();
    // ---- C: delta rule update, o = Qn . S ----
    const float kvv = (red_kv[0][c] + red_kv[1][c]) + (red_kv[2][c] + red_kv[3][c]);
    const float delta = (v_t - kvv) * bt;
    float po = 0.f;
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      s[i] = fmaf(kn_s[rq * RPW + i], delta, s[i]);
      po = fmaf(s[i], qn_s[rq * RPW + i], po);
    }
    red_o[rq][c] = po;
    __syncthreads();
    // ---- D: output column (row-quarter-0 warps) ----
    if (rq == 0) {
      const float o = (red_o[0][c] + red_o[1][c]) + (red_o[2][c] + red_o[3][c]);
      if (a.core) a.core[base * DV + c] = o;
      if constexpr (FUSED) {
        const float sq = warp_sum(o * o);
        if (lane == 0) ss_s[cgp] = sq;
        o_prev = o;
        z_prev = z_t;
        out_prev = base * DV + c;
      }
    }
  }
  if (FUSED && a.S) {
    __syncthreads();
    if (rq == 0) {
      const float inv = 1.0f / sqrtf((ss_s[0] + ss_s[1] + ss_s[2] + ss_s[3]) / (float)DV + a.eps);
      a.y[out_prev] = gam * (o_prev * inv) * (z_prev / (1.0f + expf(-z_prev)));
    }
  }
  if (a.state_out) {
#pragma unroll
    for (int i = 0; i < RPW; ++i) a.state_out[sbase + (uint64_t)(rq * RPW + i) * DV + c] = s[i];
  }
}

// Decode-length variant (a few tokens per call) of the head-per-CTA recurrence: thread = warp w's
// rows [8w, 8w+8) x lane's columns [4*lane, 4*lane+4), so the state moves as eight float4 loads
// and stores per thread (the scalar layout above issues 32 of each and is load/store-queue bound
// when one launch is one token).  Reductions over dk sum 16 row-group partials per column from
// shared memory; warp 0 holds all 128 columns of the output and finishes the gated norm alone.
template <bool FUSED>
__global__ void __launch_bounds__(512) deltanet_head_vec_kernel(DeltaArgs a) {
  constexpr int DK = 128, DV = 128, R = 8;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t h = blockIdx.x, hk = h % a.HK;
  const int c0 = lane * 4, r0 = warp * R;
  __shared__ float kn_s[DK], qn_s[DK];
  __shared__ __align__(16) float red_kv[16][DV], red_o[16][DV];

  float kq[4], ga, gb;
  float4 vv, zz = make_float4(0.f, 0.f, 0.f, 0.f);
  auto load_inputs = [&](uint32_t t) {
    const uint32_t tt = t + a.tOff;
    const uint64_t base = (uint64_t)tt * a.H + h, basek = (uint64_t)tt * a.HK + hk;
    if (warp < 2) {
      const float4 x = *reinterpret_cast<const float4 *>((warp ? a.q : a.k) + basek * DK + lane * 4);
      kq[0] = x.x; kq[1] = x.y; kq[2] = x.z; kq[3] = x.w;
    }
    vv = *reinterpret_cast<const float4 *>(a.v + base * DV + c0);
    if constexpr (FUSED) {
      if (warp == 0) zz = *reinterpret_cast<const float4 *>(a.z + base * DV + c0);
      ga = a.a[base];
      gb = a.b[base];
    } else {
      ga = a.g[base];
      gb = a.beta[a.betaOff + base];
    }
  };
  if (a.S) load_inputs(0);

  float s[R][4];
  const uint64_t sbase = (uint64_t)h * DK * DV;
#pragma unroll
  for (int i = 0; i < R; ++i) {
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (a.loadState && a.state_in)
      x = *reinterpret_cast<const float4 *>(a.state_in + sbase + (uint64_t)(r0 + i) * DV + c0);
    s[i][0] = x.x; s[i][1] = x.y; s[i][2] = x.z; s[i][3] = x.w;
  }
  const float qscale = 1.0f / sqrtf((float)DK);
  const float an = FUSED ? a.a_neg[h] : 0.f, dtb = FUSED ? a.dt_bias[h] : 0.f;
  float4 gam = make_float4(0.f, 0.f, 0.f, 0.f);
  if (FUSED && warp == 0) gam = *reinterpret_cast<const float4 *>(a.gamma + c0);

  for (uint32_t t = 0; t < a.S; ++t) {
    const uint64_t base = (uint64_t)(t + a.tOff) * a.H + h;
    if (warp < 2) {  // l2norm(k), l2norm(q)/sqrt(dk)
      float ss = kq[0] * kq[0] + kq[1] * kq[1] + kq[2] * kq[2] + kq[3] * kq[3];
      ss = warp_sum(ss);
      const float inv = (1.0f / sqrtf(ss + 1e-6f)) * (warp ? qscale : 1.0f);
      float *dst = (warp ? qn_s : kn_s) + lane * 4;
      dst[0] = kq[0] * inv; dst[1] = kq[1] * inv; dst[2] = kq[2] * inv; dst[3] = kq[3] * inv;
    }
    float gt, bt;
    if constexpr (FUSED) {
      gt = expf(an * softplus_stable(ga + dtb));
      bt = sigmoidf_(gb);
    } else {
      gt = expf(ga);
      bt = gb;
    }
    const float vt[4] = {vv.x, vv.y, vv.z, vv.w};
    const float zt[4] = {zz.x, zz.y, zz.z, zz.w};
    if (t + 1 < a.S) load_inputs(t + 1);
    __syncthreads();
    float kn[R], qn[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      kn[i] = kn_s[r0 + i];
      qn[i] = qn_s[r0 + i];
    }
    float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < R; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        s[i][c] *= gt;
        part[c] = fmaf(s[i][c], kn[i], part[c]);
      }
    *reinterpret_cast<float4 *>(&red_kv[warp][c0]) = make_float4(part[0], part[1], part[2], part[3]);
    __syncthreads();
    float kvv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < 16; ++w) {
      const float4 x = *reinterpret_cast<const float4 *>(&red_kv[w][c0]);
      kvv[0] += x.x; kvv[1] += x.y; kvv[2] += x.z; kvv[3] += x.w;
    }
    float po[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float delta = (vt[c] - kvv[c]) * bt;
#pragma unroll
      for (int i = 0; i < R; ++i) {
        s[i][c] = fmaf(kn[i], delta, s[i][c]);
        po[c] = fmaf(s[i][c], qn[i], po[c]);
      }
    }
    *reinterpret_cast<float4 *>(&red_o[warp][c0]) = make_float4(po[0], po[1], po[2], po[3]);
    __syncthreads();
    if (warp == 0) {
      float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int w = 0; w < 16; ++w) {
        const float4 x = *reinterpret_cast<const float4 *>(&red_o[w][c0]);
        o[0] += x.x; o[1] += x.y; o[2] += x.z; o[3] += x.w;
      }
      if (a.core) *reinterpret_cast<float4 *>(a.core + base * DV + c0) = make_float4(o[0], o[1], o[2], o[3]);
      if constexpr (FUSED) {
        const float sq = warp_sum(o[0] * o[0] + o[1] * o[1] + o[2] * o[2] + o[3] * o[3]);
        const float inv = 1.0f / sqrtf(sq / (float)DV + a.eps);
        const float g4[4] = {gam.x, gam.y, gam.z, gam.w};
        float y[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) y[c] = g4[c] * (o[c] * inv) * (zt[c] / (1.0f + expf(-zt[c])));
        *reinterpret_cast<float4 *>(a.y + base * DV + c0) = make_float4(y[0], y[1], y[2], y[3]);
      }
    }
  }
  if (a.state_out) {
#pragma unroll
    for (int i = 0; i < R; ++i)
      *reinterpret_cast<float4 *>(a.state_out + sbase + (uint64_t)(r0 + i) * DV + c0) =
          make_float4(s[i][0], s[i][1], s[i][2], s[i][3]);
  }
}

// Decode (calls of at most 16 tokens) for DK = DV = 128: the state columns of a head split over a
// cluster of kSplitCTAs CTAs (kSplitCols columns each), so a 48-head layer runs 384 CTAs across all
// SMs instead of 48 and each SM moves ~1/148 of the state.  Thread (row group rg, column group cg)
// holds rows [4 rg, 4 rg + 4) x columns [4 cg, 4 cg + 4) of the CTA's slice: the state moves as
// four float4 loads and stores per thread.  The two reductions over dk per token run as warp
// shuffles plus one shared-memory pass over the CTA's warps; the gated norm's sum of squares over
// all 128 columns crosses the cluster one way: every CTA stores its partial into each peer's
// shared memory with st.async, which counts the bytes on the peer's mbarrier, and waits on its own
// mbarrier for all partials (double-buffered by token parity) -- no cluster-wide barrier per token.
template <bool FUSED, int NC>
__global__ void __launch_bounds__(NC * 8) deltanet_split_kernel(DeltaArgs a) {
  constexpr int DK = 128, DV = 128, CG = NC / 4, NT = NC * 8, NW = NT / 32, kSplitCTAs = 128 / NC;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cg_ = tid % CG, rg = tid / CG;           // 32 row groups of 4 rows
  const uint32_t split = blockIdx.x, h = blockIdx.y, hk = h % a.HK;
  const int r0 = 4 * rg, col = (int)split * NC + 4 * cg_;
  // Programmatic dependent launch: let the next kernel of the stream get scheduled now; it waits
  // in its own griddepcontrol.wait until this grid has completed and its writes are visible.
  // Nothing is read before this grid's own wait (the previous kernel may produce any input,
  // the state included).
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // While the previous kernel may still run, warm L2 with this thread's state rows: a prefetch
  // returns no data, and L2 stays coherent with whatever that kernel writes, so this is safe.
  if (a.loadState && a.state_in && a.S) {
    const float *sp = a.state_in + (uint64_t)h * 128 * 128 + (uint64_t)r0 * 128 + col;
#pragma unroll
    for (int i = 0; i < 4; ++i) asm volatile("prefetch.global.L2 [%0];" ::"l"(sp + i * 128));
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ __align__(16) float kn_s[DK], qn_s[DK];
  __shared__ __align__(16) float red_kv[NW][NC], red_o[NW][NC];
  __shared__ float ss_in[2][8];                 // partial sums of squares from each cluster rank
  __shared__ __align__(8) uint64_t ss_bar[2];   // their arrival, by token parity
  uint32_t my_rank = 0;
  if constexpr (FUSED) {
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(my_rank));
    if (tid == 0) {
      mbar_init(&ss_bar[0], 1);
      mbar_init(&ss_bar[1], 1);
      fence_barrier_init();
    }
    // peers may store into this CTA only after its barriers exist: arrive now, wait before the
    // first exchange (the state loads in between hide the barrier latency)
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  }

  float kq[4] = {0.f, 0.f, 0.f, 0.f}, ga = 0.f, gb = 0.f;
  float4 vv = make_float4(0.f, 0.f, 0.f, 0.f), zz = vv;
  auto load_inputs = [&](uint32_t t) {
    const uint32_t tt = t + a.tOff;
    const uint64_t base = (uint64_t)tt * a.H + h, basek = (uint64_t)tt * a.HK + hk;
    if (warp < 2) {
      const float4 x = *reinterpret_cast<const float4 *>((warp ? a.q : a.k) + basek * DK + lane * 4);
      kq[0] = x.x; kq[1] = x.y; kq[2] = x.z; kq[3] = x.w;
    }
    vv = *reinterpret_cast<const float4 *>(a.v + base * DV + col);
    if constexpr (FUSED) {
      if (rg == 0) zz = *reinterpret_cast<const float4 *>(a.z + base * DV + col);
      ga = a.a[base];
      gb = a.b[base];
    } else {
      ga = a.g[base];
      gb = a.beta[a.betaOff + base];
    }
  };
  if (a.S) load_inputs(0);
  float s[4][4];
  const uint64_t sbase = (uint64_t)h * DK * DV;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (a.loadState && a.state_in) x = *reinterpret_cast<const float4 *>(a.state_in + sbase + (uint64_t)(r0 + i) * DV + col);
    s[i][0] = x.x; s[i][1] = x.y; s[i][2] = x.z; s[i][3] = x.w;
  }
  const float qscale = 1.0f / sqrtf((float)DK);
  const float an = FUSED ? a.a_neg[h] : 0.f, dtb = FUSED ? a.dt_bias[h] : 0.f;
  float4 gam = make_float4(0.f, 0.f, 0.f, 0.f);
  if (FUSED && rg == 0) gam = *reinterpret_cast<const float4 *>(a.gamma + col);

  // sum over the CTA's rows of per-thread partials p[4] for its 4 columns -> full sums, every thread
  auto row_sum = [&](float (&p)[4], float (*red)[NC]) {
#pragma unroll
    for (int o = CG; o < 32; o <<= 1)
#pragma unroll
      for (int c = 0; c < 4; ++c) p[c] += __shfl_xor_sync(0xffffffffu, p[c], o);
    if (lane < CG) *reinterpret_cast<float4 *>(&red[warp][4 * lane]) = make_float4(p[0], p[1], p[2], p[3]);
    __syncthreads();
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float4 x = *reinterpret_cast<const float4 *>(&red[w][4 * cg_]);
      acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
    }
    p[0] = acc.x; p[1] = acc.y; p[2] = acc.z; p[3] = acc.w;
  };

  for (uint32_t t = 0; t < a.S; ++t) {
    const uint64_t base = (uint64_t)(t + a.tOff) * a.H + h;
    if (warp < 2) {  // l2norm(k), l2norm(q)/sqrt(dk)
      float ss = kq[0] * kq[0] + kq[1] * kq[1] + kq[2] * kq[2] + kq[3] * kq[3];
      ss = warp_sum(ss);
      const float inv = (1.0f / sqrtf(ss + 1e-6f)) * (warp ? qscale : 1.0f);
      *reinterpret_cast<float4 *>((warp ? qn_s : kn_s) + lane * 4) =
          make_float4(kq[0] * inv, kq[1] * inv, kq[2] * inv, kq[3] * inv);
    }
    float gt, bt;
    if constexpr (FUSED) {
      gt = expf(an * softplus_stable(ga + dtb));
      bt = sigmoidf_(gb);
    } else {
      gt = expf(ga);
      bt = gb;
    }
    const float vt[4] = {vv.x, vv.y, vv.z, vv.w};
    const float zt[4] = {zz.x, zz.y, zz.z, zz.w};
    if (t + 1 < a.S) load_inputs(t + 1);
    __syncthreads();
    const float4 kn4 = *reinterpret_cast<const float4 *>(kn_s + r0);
    const float4 qn4 = *reinterpret_cast<const float4 *>(qn_s + r0);
    const float kn[4] = {kn4.x, kn4.y, kn4.z, kn4.w}, qn[4] = {qn4.x, qn4.y, qn4.z, qn4.w};
    float kv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        s[i][c] *= gt;
        kv[c] = fmaf(s[i][c], kn[i], kv[c]);
      }
    row_sum(kv, red_kv);
    float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float delta = (vt[c] - kv[c]) * bt;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        s[i][c] = fmaf(kn[i], delta, s[i][c]);
        o[c] = fmaf(s[i][c], qn[i], o[c]);
      }
    }
    row_sum(o, red_o);
    if constexpr (FUSED) {
      if (t == 0) asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
      const int slot = t & 1;
      if (warp == 0) {
        float sq = lane < CG ? o[0] * o[0] + o[1] * o[1] + o[2] * o[2] + o[3] * o[3] : 0.f;
        sq = warp_sum(sq);
        if (lane == 0) mbar_expect_tx(&ss_bar[slot], 4 * kSplitCTAs);
        if (lane < kSplitCTAs) {  // lane r stores this CTA's partial into rank r
          uint32_t raddr, rbar;
          asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(raddr) : "r"(smem_u32(&ss_in[slot][my_rank])), "r"(lane));
          asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbar) : "r"(smem_u32(&ss_bar[slot])), "r"(lane));
          asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr),
                       "r"(__float_as_uint(sq)), "r"(rbar)
                       : "memory");
        }
      }
      if (rg == 0) {
        float tot = 0.f;
        if (mbar_wait(&ss_bar[slot], (t >> 1) & 1)) {
#pragma unroll
          for (int r = 0; r < kSplitCTAs; ++r) tot += ss_in[slot][r];
        }
        const float inv = 1.0f / sqrtf(tot / (float)DV + a.eps);
        const float g4[4] = {gam.x, gam.y, gam.z, gam.w};
        float y[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) y[c] = g4[c] * (o[c] * inv) * (zt[c] / (1.0f + expf(-zt[c])));
        *reinterpret_cast<float4 *>(a.y + base * DV + col) = make_float4(y[0], y[1], y[2], y[3]);
      }
    }
    if (rg == 0 && a.core) *reinterpret_cast<float4 *>(a.core + base * DV + col) = make_float4(o[0], o[1], o[2], o[3]);
    // red_kv / red_o are rewritten by the next token only after its first block barrier
  }
  // A CTA leaves only after its threads of row group 0 received every peer's last partial, so no
  // store into its shared memory is still on the way.  (S == 0: the startup barrier still pairs.)
  if (FUSED && a.S == 0) asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (a.state_out) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      *reinterpret_cast<float4 *>(a.state_out + sbase + (uint64_t)(r0 + i) * DV + col) =
          make_float4(s[i][0], s[i][1], s[i][2], s[i][3]);
  }
}

}  // namespace

int poll_device_error_deltanet() {
  int v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return BG_ELAUNCH;
  if (v) cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
  return v;
}

namespace {

__global__ void gbeta_kernel(const float *a, const float *b, const float *an, const float *dt, uint32_t S, uint32_t H,
                             float *out) {
  const uint32_t n = S * H;
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t h = i % H;
  out[i] = an[h] * softplus_stable(a[i] + dt[h]);
  out[n + i] = sigmoidf_(b[i]);
}

// one warp per row (deltanet_norm_gate.wgsl:19-31)
__global__ void norm_gate_kernel(const float *core, const float *z, const float *gamma, uint32_t rows, uint32_t DV,
                                 float eps, float *y) {
  const uint32_t row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float *cr = core + (uint64_t)row * DV;
  float ss = 0.f;
  for (uint32_t i = lane; i < DV; i += 32) ss = fmaf(cr[i], cr[i], ss);
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / (float)DV + eps);
  for (uint32_t i = lane; i < DV; i += 32) {
    const float zz = z[(uint64_t)row * DV + i];
    y[(uint64_t)row * DV + i] = gamma[i] * (cr[i] * inv) * (zz / (1.0f + expf(-zz)));
  }
}

__global__ void gate_sigmoid_kernel(const float *x, const float *g, uint32_t n, float *y) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = x[i] / (1.0f + expf(-g[i]));
}

constexpr uint32_t kVecMaxTokens = 16;

// the vector layout reads state, q/k, v, z, gamma and writes state, core, y as float4
bool aligned16(const DeltaArgs &a) {
  const void *ps[] = {a.state_in, a.state_out, a.q, a.k, a.v, a.z, a.gamma, a.core, a.y};
  for (const void *x : ps)
    if (reinterpret_cast<uintptr_t>(x) % 16) return false;
  return true;
}

// BGATTN_PDL=0 launches the decode kernel without programmatic dependent launch (A/B checks)
bool pdl_enabled() {
  static const bool v = [] {
    const char *e = getenv("BGATTN_PDL");
    return !(e && *e == '0');
  }();
  return v;
}

// columns per CTA of the split decode kernel: 16 (8-CTA clusters, default) or 32 (BGATTN_DN_COLS=32)
int dn_split_cols() {
  static const int v = [] {
    const char *e = getenv("BGATTN_DN_COLS");
    return (e && atoi(e) == 32) ? 32 : 16;
  }();
  return v;
}

// BGATTN_DN_SPLIT=0 keeps decode on the one-CTA-per-head vector kernel (A/B checks)
bool dn_split_enabled() {
  static const bool v = [] {
    const char *e = getenv("BGATTN_DN_SPLIT");
    return !(e && *e == '0');
  }();
  return v;
}

bool head_legacy() {
  static const bool v = [] {
    const char *e = getenv("BGATTN_DN_LEGACY");  // column-group kernel with the cluster norm (A/B)
    return e && *e == '1';
  }();
  return v;
}

template <int DK>
int launch_dk(const DeltaArgs &a, cudaStream_t st) {
  const uint32_t ncg = (a.DV + 31) / 32;
  const bool fused = a.z != nullptr;
  if (DK == 128 && a.DV == 128 && !head_legacy()) {
    // short calls (decode) take the vector layout; long recurrent runs keep the scalar one, whose
    // per-token reductions are four partials instead of sixteen
    const bool vec = a.S <= kVecMaxTokens && aligned16(a);
    if (vec && dn_split_enabled()) {
      const int nc = dn_split_cols();
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(128 / nc, a.H);
      cfg.blockDim = dim3(nc * 8);
      cfg.stream = st;
      cudaLaunchAttribute attr[2];
      int na = 0;
      attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[na++].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
      if (fused) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 128 / nc;
        attr[na].val.clusterDim.y = 1;
        attr[na++].val.clusterDim.z = 1;
      }
      cfg.attrs = attr;
      cfg.numAttrs = na;
      cudaError_t e;
      if (nc == 32) e = fused ? cudaLaunchKernelEx(&cfg, deltanet_split_kernel<true, 32>, a)
                              : cudaLaunchKernelEx(&cfg, deltanet_split_kernel<false, 32>, a);
      else e = fused ? cudaLaunchKernelEx(&cfg, deltanet_split_kernel<true, 16>, a)
                     : cudaLaunchKernelEx(&cfg, deltanet_split_kernel<false, 16>, a);
      return e == cudaSuccess ? BG_OK : BG_ELAUNCH;
    }
    if (vec && fused) deltanet_head_vec_kernel<true><<<a.H, 512, 0, st>>>(a);
    else if (vec) deltanet_head_vec_kernel<false><<<a.H, 512, 0, st>>>(a);
    else if (fused) deltanet_head_kernel<true><<<a.H, 512, 0, st>>>(a);
    else deltanet_head_kernel<false><<<a.H, 512, 0, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
  }
  if (!fused) {
    deltanet_kernel<DK, false><<<dim3(ncg, a.H), 128, 0, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
  }
  if (ncg > 8) return BG_EUNSUPPORTED;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ncg, a.H);
  cfg.blockDim = dim3(128);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = ncg;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, deltanet_kernel<DK, true>, a);
  return e == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

}  // namespace

int launch_deltanet(const DeltaArgs &a, cudaStream_t st) {
  if (a.S == 0) return BG_OK;
  switch (a.DK) {
    case 64: return launch_dk<64>(a, st);
    case 128: return launch_dk<128>(a, st);
    default: return BG_EUNSUPPORTED;
  }
}

int launch_gbeta(const float *a, const float *b, const float *an, const float *dt, uint32_t S, uint32_t H, float *out,
                 cudaStream_t st) {
  const uint32_t n = S * H;
  if (!n) return BG_OK;
  gbeta_kernel<<<(n + 255) / 256, 256, 0, st>>>(a, b, an, dt, S, H, out);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

int launch_norm_gate(const float *core, const float *z, const float *gamma, uint32_t rows, uint32_t DV, float eps,
                     float *y, cudaStream_t st) {
  if (!rows) return BG_OK;
  norm_gate_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>(core, z, gamma, rows, DV, eps, y);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

int launch_gate_sigmoid(const float *x, const float *g, uint32_t n, float *y, cudaStream_t st) {
  if (!n) return BG_OK;
  gate_sigmoid_kernel<<<(n + 255) / 256, 256, 0, st>>>(x, g, n, y);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}

}  // namespace bg
