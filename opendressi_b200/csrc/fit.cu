// 2-D image fitting step (config C1): the whole reference graph
//   loss = Mean((param - target)^2)          (examples/image_fitting/run.cpp:47)
//   g    = BuildBackward(loss)               (per texel: c*diff + c*diff)
//   in-graph Adam on param                   (silhouette example run.cpp:421-436)
// as ONE memory-bound pass: each texel is read once (param, target, m, v)
// and written once (param, m, v) -- 112 B/texel, float4-vectorised.
//
// The Adam counter lives on the device: every block reads t, computes
// t_new = t + 1 and the bias corrections itself; the last block to finish
// (completion ticket) publishes t_new and the loss, so the step needs no
// host round trip and can be replayed from a CUDA graph.
#include <algorithm>

#include "kernels.h"

namespace dressi {

__global__ void __launch_bounds__(256)
        k_fit_step(size_t n4, float lr, float inv_n, FitBuffers b) {
    const float b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
    const float omb1 = 1.f - b1, omb2 = 1.f - b2;
    const float t_new = b.scalars[0] + 1.f;
    const float bc1 = 1.f - powf(b1, t_new);
    const float bc2 = 1.f - powf(b2, t_new);
    const float g_sq = 1.f * inv_n;
    double acc = 0.0;
    float4* P = reinterpret_cast<float4*>(b.param);
    const float4* T = reinterpret_cast<const float4*>(b.target);
    float4* M = reinterpret_cast<float4*>(b.m);
    float4* V = reinterpret_cast<float4*>(b.v);
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += size_t(gridDim.x) * blockDim.x) {
        float4 p = P[i];
        const float4 t = T[i];
        float4 m = M[i], v = V[i];
        float* pp = &p.x;
        const float* tp = &t.x;
        float* mp = &m.x;
        float* vp = &v.x;
        float part = 0.f;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const float diff = pp[c] - tp[c];
            part += diff * diff;
            const float g = g_sq * diff + g_sq * diff;
            const float m_new = mp[c] * b1 + g * omb1;
            const float v_new = vp[c] * b2 + g * g * omb2;
            const float step = (m_new / bc1) / (sqrtf(v_new / bc2) + eps) * lr;
            pp[c] = pp[c] - step;
            mp[c] = m_new;
            vp[c] = v_new;
        }
        acc += part;
        P[i] = p;
        M[i] = m;
        V[i] = v;
    }
    __shared__ double red[8];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    __shared__ bool last;
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int w = 0; w < 8; w++) s += red[w];
        atomicAdd(b.loss_acc, s);
        __threadfence();
        last = atomicAdd(b.done, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        __threadfence();
        const double total = atomicAdd(b.loss_acc, 0.0);
        const float loss = float(total * double(inv_n));
        b.scalars[3] = loss;
        const int it = int(t_new) - 1;
        if (b.hist_cap > 0) b.loss_hist[it % b.hist_cap] = loss;
        b.scalars[0] = t_new;
        *b.loss_acc = 0.0;
        *b.done = 0u;
    }
}

void fit_iteration(size_t n, float lr, const FitBuffers& b, cudaStream_t s) {
    const size_t n4 = n / 4;
    int dev = 0, sms = 148;
    DRESSI_CUDA(cudaGetDevice(&dev));
    DRESSI_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int blocks = int(std::max<size_t>(
            1, std::min<size_t>((n4 + 255) / 256, size_t(sms) * 8)));
    ProfScope ps("fit_step", s);
    k_fit_step<<<blocks, 256, 0, s>>>(n4, lr, 1.f / float(n), b);
    DRESSI_CUDA(cudaGetLastError());
}

}  // namespace dressi
