// Hard rasterizer (F::RasterizeFaceId / F::Rasterize): tile-binned and
// bit-exact with the reference's RasterizeCore (cpu_raster.cpp:31-110).
//
// The reference keeps, per pixel, the fragment with the smallest NDC z and
// the latest face on ties (`if (z > zb) continue;`). Each thread owns two
// pixels and folds every fragment of its tile's face list into their keys,
// so list order does not matter. The survivor's barycentrics are recomputed
// once at the end for the attribute interpolation, with the reference's
// expressions (shade lambda, cpu_raster.cpp:205-223).
#include <algorithm>
#include <cstdlib>

#include "kernels.h"

namespace dressi {

struct __align__(16) HardRec {
    float x0, y0, x1, y1;   // screen px
    float x2, y2, inv_area, zlb;  // zlb: lower bound of every fragment depth
    float z0, z1, z2, pad2;  // NDC depth
    float iw0, iw1, iw2, pad3;  // 1 / clip.w
    int bx0, bx1, by0, by1;  // pixel range (inclusive)
    uint32_t flags, i0, i1, i2;
};
static_assert(sizeof(HardRec) == 96, "HardRec layout");
constexpr int kHardVec4 = sizeof(HardRec) / 16;

struct HardBuffers {
    HardRec* recs;
    BinSet bin;
    uint32_t* status;
};

static void carve_hard(Arena& a, const HardDims& d, HardBuffers* b) {
    const size_t vt = size_t(d.views) * d.n_tiles;
    b->recs = a.take<HardRec>(size_t(d.views) * std::max(d.n_faces, 1));
    b->bin.count = a.take<int>(vt);
    b->bin.offset = a.take<int>(vt);
    b->bin.cursor = a.take<int>(vt);
    b->bin.overflow = a.take<int>(d.views);
    b->bin.cap = d.cap;
    b->bin.list = a.take<int>(size_t(d.views) * d.cap);
}

static HardDims with_cap(HardDims d) {
    d.finalize();
    if (d.cap <= 0) {
        const long long f = d.n_faces, t = d.n_tiles;
        d.cap = int(std::min<long long>(std::max<long long>(16 * f, 4 * t) + 4096,
                                        1ll << 30));
        // test hook shared with the soft rasterizer (exercises the fallback)
        if (const char* e = std::getenv("DRESSI_B200_BIN_CAP")) {
            const long long c = std::atoll(e);
            if (c > 0) d.cap = int(std::min<long long>(c, 1ll << 30));
        }
    }
    return d;
}

size_t hard_workspace_bytes(const HardDims& d0) {
    const HardDims d = with_cap(d0);
    Arena a;
    HardBuffers b;
    carve_hard(a, d, &b);
    return a.used + 256;
}

// RasterizeCore's per-face prologue (cpu_raster.cpp:43-78).
__global__ void k_hard_setup(HardDims d, const float4* clip,
                             const float* faces, HardBuffers b) {
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    const int v = blockIdx.y;
    if (f >= d.n_faces) return;
    HardRec r;
    r.flags = 0;
    uint32_t idx[3];
    float sx[3], sy[3], sz[3], iw[3];
    bool ok = true;
    for (int k = 0; k < 3; k++) {
        idx[k] = x86_u32_via_i64(faces[size_t(f) * 3 + k]);
        if (idx[k] >= uint32_t(d.n_verts)) {
            atomicOr(b.status, kStatusIndexRange);
            ok = false;
            break;
        }
        const float4 c = clip[size_t(v) * d.n_verts + idx[k]];
        if (fabsf(c.w) <= 1e-6f || c.w < 0.f) {
            ok = false;
            break;
        }
        const float inv_w = 1.f / c.w;
        sx[k] = (c.x * inv_w * 0.5f + 0.5f) * float(d.W);
        sy[k] = (c.y * inv_w * 0.5f + 0.5f) * float(d.H);
        sz[k] = c.z * inv_w;
        iw[k] = inv_w;
    }
    if (ok) {
        const float area = (sx[1] - sx[0]) * (sy[2] - sy[0]) -
                           (sy[1] - sy[0]) * (sx[2] - sx[0]);
        if (!(fabsf(area) < 1e-6f)) {
            r.x0 = sx[0]; r.y0 = sy[0]; r.x1 = sx[1]; r.y1 = sy[1];
            r.x2 = sx[2]; r.y2 = sy[2];
            r.inv_area = 1.f / area;
            r.z0 = sz[0]; r.z1 = sz[1]; r.z2 = sz[2];
            r.iw0 = iw[0]; r.iw1 = iw[1]; r.iw2 = iw[2];
            r.pad2 = r.pad3 = 0.f;
            // A covered pixel has computed l_k >= 0 whose sum is within
            // 3u of 1 (u = 2^-24; l2 = 1 - l0 - l1 takes two roundings), so
            // sum(l_k z_k) >= zmin - 3u max|z_k|, and evaluating it takes 5
            // more roundings (<= 5u (1 + 3u) max|z_k|): the fragment depth is
            // at least zmin - 8u max|z_k|; 1e-6 (~16.8u) covers it.
            const float zmin = std_min(std_min(sz[0], sz[1]), sz[2]);
            const float zabs = fmaxf(fmaxf(fabsf(sz[0]), fabsf(sz[1])), fabsf(sz[2]));
            r.zlb = zmin - 1e-6f * zabs;
            if (!(r.zlb == r.zlb)) r.zlb = -INFINITY;  // NaN: never skipped
            bbox_range(std_min(std_min(sx[0], sx[1]), sx[2]),
                       std_max(std_max(sx[0], sx[1]), sx[2]), d.W, &r.bx0,
                       &r.bx1);
            bbox_range(std_min(std_min(sy[0], sy[1]), sy[2]),
                       std_max(std_max(sy[0], sy[1]), sy[2]), d.H, &r.by0,
                       &r.by1);
            r.i0 = idx[0]; r.i1 = idx[1]; r.i2 = idx[2];
            if (r.bx0 <= r.bx1 && r.by0 <= r.by1) r.flags = kFaceValid;
        }
    }
    b.recs[size_t(v) * d.n_faces + f] = r;
    if (!(r.flags & kFaceValid)) return;
    int tx0, tx1, ty0, ty1;
    tile_range(r.bx0, r.bx1, r.by0, r.by1, &tx0, &tx1, &ty0, &ty1);
    int* cnt = b.bin.count + size_t(v) * d.n_tiles;
    for (int ty = ty0; ty <= ty1; ty++)
        for (int tx = tx0; tx <= tx1; tx++) atomicAdd(&cnt[ty * d.tiles_x + tx], 1);
}

__global__ void k_hard_fill(HardDims d, HardBuffers b) {
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    const int v = blockIdx.y;
    if (f >= d.n_faces) return;
    const HardRec& r = b.recs[size_t(v) * d.n_faces + f];
    if (!(r.flags & kFaceValid)) return;
    const bool of = b.bin.overflow[v] != 0;
    int tx0, tx1, ty0, ty1;
    tile_range(r.bx0, r.bx1, r.by0, r.by1, &tx0, &tx1, &ty0, &ty1);
    int* cur = b.bin.cursor + size_t(v) * d.n_tiles;
    int* list = b.bin.list + size_t(v) * b.bin.cap;
    for (int ty = ty0; ty <= ty1; ty++)
        for (int tx = tx0; tx <= tx1; tx++) {
            const int slot = atomicAdd(&cur[ty * d.tiles_x + tx], 1);
            if (!of && slot < b.bin.cap) list[slot] = f;
        }
}

// Screen barycentrics of RasterizeCore (cpu_raster.cpp:82-90).
__device__ __forceinline__ void hard_bary(const HardRec& r, float px, float py,
                                          float* l0, float* l1, float* l2) {
    *l0 = ((r.x1 - px) * (r.y2 - py) - (r.y1 - py) * (r.x2 - px)) * r.inv_area;
    *l1 = ((r.x2 - px) * (r.y0 - py) - (r.y2 - py) * (r.x0 - px)) * r.inv_area;
    *l2 = 1.f - *l0 - *l1;
}

// Order-preserving key of a float (ascending floats -> ascending keys).
__device__ __forceinline__ unsigned long long zlb_key(float z) {
    const uint32_t u = __float_as_uint(z);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// The float of a zlb_key.
__device__ __forceinline__ float zlb_of_key(unsigned long long k) {
    const uint32_t u = uint32_t(k >> 32);
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

// The outputs of one pixel from its survivor (best_f < 0: background).
__device__ __forceinline__ void hard_out(const HardDims& d, const float* attr,
                                         float* out, float* depth_out,
                                         float* id_out, const HardRec* recs,
                                         int v, int x, int y, bool in,
                                         float best_z, int best_f) {
    const float px = float(x) + 0.5f, py = float(y) + 0.5f;
    if (!in) return;
    const size_t pix = size_t(v) * d.W * d.H + size_t(y) * d.W + x;
    if (depth_out) depth_out[pix] = best_f >= 0 ? best_z : 1.f;
    if (id_out) id_out[pix] = best_f >= 0 ? float(best_f) + 1.f : 0.f;
    if (d.uvzw) {
        // The reference's rasterize (python/dressi/torch/ops.py:96-110):
        // g = Rasterize(unwelded clip, corner attributes), tid =
        // RasterizeFaceId, z/w = g.z / (g.w + (1 - mask)).
        float4* o4 = reinterpret_cast<float4*>(out) + pix;
        if (best_f < 0) {
            *o4 = make_float4(0.f, 0.f, 0.f / (0.f + 1.f), 0.f);
            return;
        }
        const HardRec& r = recs[best_f];
        float l[3];
        hard_bary(r, px, py, &l[0], &l[1], &l[2]);
        const float iw[3] = {r.iw0, r.iw1, r.iw2};
        const uint32_t idx[3] = {r.i0, r.i1, r.i2};
        const float denom = l[0] * iw[0] + l[1] * iw[1] + l[2] * iw[2];
        const float4* pg = reinterpret_cast<const float4*>(attr) + size_t(v) * d.n_verts;
        float num[4] = {0.f, 0.f, 0.f, 0.f};
        for (int k = 0; k < 3; k++) {
            const float4 a = pg[idx[k]];
            const float ak[4] = {k == 0 ? 1.f : 0.f, k == 1 ? 1.f : 0.f, a.z, a.w};
            for (int c = 0; c < 4; c++) num[c] += l[k] * iw[k] * ak[c];
        }
        const float gz = num[2] / denom, gw = num[3] / denom;
        *o4 = make_float4(num[0] / denom, num[1] / denom, gz / (gw + (1.f - 1.f)),
                          float(best_f) + 1.f);
        return;
    }
    if (!attr && !d.attr_ones) {
        out[pix] = best_f >= 0 ? float(best_f) + 1.f : 0.f;
        return;
    }
    float* o = out + pix * d.n_comp;
    if (best_f < 0) {
        for (int c = 0; c < d.n_comp; c++) o[c] = 0.f;
        return;
    }
    const HardRec& r = recs[best_f];
    float l[3];
    hard_bary(r, px, py, &l[0], &l[1], &l[2]);
    const float iw[3] = {r.iw0, r.iw1, r.iw2};
    const uint32_t idx[3] = {r.i0, r.i1, r.i2};
    const float denom = l[0] * iw[0] + l[1] * iw[1] + l[2] * iw[2];
    const float* av = d.attr_ones ? nullptr
                      : attr + (d.attr_shared ? 0 : size_t(v) * d.n_verts * d.n_comp);
    for (int c = 0; c < d.n_comp; c++) {
        float num = 0.f;
        for (int k = 0; k < 3; k++)
            num += l[k] * iw[k] * (av ? av[size_t(idx[k]) * d.n_comp + c] : 1.f);
        o[c] = num / denom;
    }
}

// The sweep runs kHardWarps warps per 16x16 tile, each over a 16x4 region
// (two of the tile's 8x4 blocks, one pixel of each per lane) and on its
// own: it gathers the tile-list faces whose pixel range meets its region
// (up to kHardWin at a time), sorts them front to back by their depth lower
// bound, stages their records kHardRecs at a time in its shared slots and
// folds each lane's two pixels. With a single sorted window a pixel stops
// at the first face whose bound lies behind its survivor.
constexpr int kHardWarps = 4;
constexpr int kHardThreads = 32 * kHardWarps;
constexpr int kHardWin = 128;
constexpr int kHardRecs = 16;

__global__ void __launch_bounds__(kHardThreads)
        k_hard_sweep(HardDims d, HardBuffers b, const float* attr, float* out,
                     float* depth_out, float* id_out) {
    __shared__ HardRec sh_all[kHardWarps][kHardRecs];
    __shared__ unsigned long long keys_all[kHardWarps][kHardWin];
    const int v = blockIdx.y, tile = blockIdx.x;
    const int tx = tile % d.tiles_x, ty = tile / d.tiles_x;
    const int wq = threadIdx.x >> 5, lane = threadIdx.x & 31;
    HardRec* sh = sh_all[wq];
    unsigned long long* keys = keys_all[wq];
    // the warp's region: columns tx*16 .. +15, rows ty*16 + 4 wq .. +3;
    // pixel j of the lane: x = tx*16 + 8 j + (lane & 7), y = row + (lane >> 3)
    const int rx0 = tx * kTile, ry0 = ty * kTile + 4 * wq;
    int xs[2], ys[2];
    bool ins[2];
#pragma unroll
    for (int j = 0; j < 2; j++) {
        xs[j] = rx0 + 8 * j + (lane & 7);
        ys[j] = ry0 + (lane >> 3);
        ins[j] = xs[j] < d.W && ys[j] < d.H;
    }
    const HardRec* recs = b.recs + size_t(v) * d.n_faces;
    const bool identity = b.bin.overflow[v] != 0;
    const int tl = v * d.n_tiles + tile;
    const int beg = identity ? 0 : b.bin.offset[tl];
    const int end = identity ? d.n_faces : b.bin.cursor[tl];
    const int* list = b.bin.list + size_t(v) * b.bin.cap;
    const unsigned lt = (1u << lane) - 1u;
    float best_z[2] = {1.f, 1.f};
    int best_f[2] = {-1, -1};
    int pos = beg;
    bool first = true;
    while (pos < end) {
        // next window: up to kHardWin entries meeting the region, in list
        // order from pos
        int n = 0;
        while (n < kHardWin && pos < end) {
            const int i = pos + lane;
            bool hit = false;
            unsigned long long k = 0ull;
            if (i < end) {
                const int f = identity ? i : list[i];
                const int4 bb = reinterpret_cast<const int4*>(recs + f)[4];
                hit = !(bb.y < rx0 || bb.x > rx0 + 15 || bb.w < ry0 ||
                        bb.z > ry0 + 3);
                if (hit)
                    k = (zlb_key(recs[f].zlb) << 32) | uint32_t(f);
            }
            const unsigned bal = __ballot_sync(0xffffffffu, hit);
            const int take = imin_(__popc(bal), kHardWin - n);
            const int slot = n + __popc(bal & lt);
            if (hit && slot < kHardWin) keys[slot] = k;
            if (take < __popc(bal)) {
                // resume at the first entry left over
                unsigned rest = bal;
                for (int t = 0; t < take; t++) rest &= rest - 1u;
                pos += __ffs(rest) - 1;
            } else {
                pos = imin_(pos + 32, end);
            }
            n += take;
        }
        __syncwarp();
        // a single window covering the whole list allows the early stop
        const bool sorted = first && pos >= end;
        first = false;
        if (n <= 32) {
            unsigned long long k = lane < n ? keys[lane] : ~0ull;
            k = warp_sort_asc(k);
            __syncwarp();
            if (lane < n) keys[lane] = k;
            __syncwarp();
        } else {
            warp_sort_smem(keys, n);
        }
        for (int base = 0; base < n; base += kHardRecs) {
            const int cn = imin_(kHardRecs, n - base);
            // the warp leaves once every pixel holds a survivor in front of
            // the next face (and so of all later ones)
            if (sorted) {
                const float zn = zlb_of_key(keys[base]);
                bool stop = true;
#pragma unroll
                for (int j = 0; j < 2; j++)
                    stop = stop && (!ins[j] || (best_f[j] >= 0 && best_z[j] < zn));
                if (__all_sync(0xffffffffu, stop)) break;
            }
            {
                const float4* src = reinterpret_cast<const float4*>(recs);
                float4* dst = reinterpret_cast<float4*>(sh);
                for (int i = lane; i < cn * kHardVec4; i += 32) {
                    const int jj = i / kHardVec4, q = i - jj * kHardVec4;
                    const int f = int(uint32_t(keys[base + jj]));
                    dst[i] = src[size_t(f) * kHardVec4 + q];
                }
                __syncwarp();
            }
            for (int t = 0; t < cn; t++) {
                const HardRec& r = sh[t];
                const int f = int(uint32_t(keys[base + t]));
                if (!(r.flags & kFaceValid)) continue;
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    if (!ins[j]) continue;
                    const int x = xs[j], y = ys[j];
                    if (x < r.bx0 || x > r.bx1 || y < r.by0 || y > r.by1) continue;
                    // every fragment of this face lies behind the survivor
                    if (best_f[j] >= 0 && r.zlb > best_z[j]) continue;
                    float l0, l1, l2;
                    hard_bary(r, float(x) + 0.5f, float(y) + 0.5f, &l0, &l1, &l2);
                    if (l0 < 0.f || l1 < 0.f || l2 < 0.f) continue;
                    const float z = l0 * r.z0 + l1 * r.z1 + l2 * r.z2;
                    if (z < 0.f || z > 1.f) continue;
                    if (beats(z, f, best_z[j], best_f[j])) {
                        best_z[j] = z;
                        best_f[j] = f;
                    }
                }
            }
            __syncwarp();  // sh reuse by the next chunk
        }
        __syncwarp();  // keys reuse by the next window
    }
#pragma unroll
    for (int j = 0; j < 2; j++)
        hard_out(d, attr, out, depth_out, id_out, recs, v, xs[j], ys[j],
                 ins[j], best_z[j], best_f[j]);
}

static void check_launch() { DRESSI_CUDA(cudaGetLastError()); }

void hard_raster_op(const HardDims& d0, void* workspace, const float* clip,
                    const float* attr, const float* faces, float* out,
                    float* depth_out, uint32_t* status, cudaStream_t s,
                    float* id_out) {
    const HardDims d = with_cap(d0);
    Arena a;
    a.base = static_cast<char*>(workspace);
    a.size = hard_workspace_bytes(d0);
    HardBuffers b;
    carve_hard(a, d, &b);
    b.status = status;
    const size_t vt = size_t(d.views) * d.n_tiles;
    DRESSI_CUDA(cudaMemsetAsync(b.bin.count, 0, vt * sizeof(int), s));
    {
        ProfScope ps("hard_bin", s);
        if (d.n_faces > 0) {
            const dim3 fg((d.n_faces + 127) / 128, d.views);
            k_hard_setup<<<fg, 128, 0, s>>>(
                    d, reinterpret_cast<const float4*>(clip), faces, b);
            k_bin_scan<<<d.views, 1024, 0, s>>>(b.bin, d.n_tiles, status);
            k_hard_fill<<<fg, 128, 0, s>>>(d, b);
        } else {
            k_bin_scan<<<d.views, 1024, 0, s>>>(b.bin, d.n_tiles, status);
        }
    }
    {
        ProfScope ps("hard_sweep", s);
        k_hard_sweep<<<dim3(d.n_tiles, d.views), kHardThreads, 0, s>>>(
                d, b, attr, out, depth_out, id_out);
    }
    check_launch();
}

// ------------------------------------------------- silhouette targets

__global__ void k_transform_plain(const float* pos, const float* mvps,
                                  int n_verts, float4* clip) {
    const int v = blockIdx.y;
    const int u = blockIdx.x * blockDim.x + threadIdx.x;
    if (u >= n_verts) return;
    clip[size_t(v) * n_verts + u] = transform_clip(
            pos[u * 3 + 0], pos[u * 3 + 1], pos[u * 3 + 2], mvps + v * 16);
}

__global__ void k_mask_from_id(float* img, size_t n) {
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += size_t(gridDim.x) * blockDim.x)
        img[i] = img[i] > 0.5f ? 1.f : 0.f;
}

void sil_transform_plain(const SilParams& p, const SilBuffers& b,
                         const float* target_pos, cudaStream_t s) {
    k_transform_plain<<<dim3((p.n_verts + 255) / 256, p.views), 256, 0, s>>>(
            target_pos, b.mvps, p.n_verts, reinterpret_cast<float4*>(b.clip));
    check_launch();
}

void sil_render_targets(const SoftDims& d, const SilParams& p,
                        const SilBuffers& b, const float* target_pos,
                        cudaStream_t s) {
    HardDims hd;
    hd.W = hd.H = p.res;
    hd.views = p.views;
    hd.n_faces = p.n_faces;
    hd.n_verts = p.n_verts;
    const size_t ws = hard_workspace_bytes(hd);
    void* mem = nullptr;
    DRESSI_CUDA(cudaMallocAsync(&mem, ws, s));
    // target clip positions go through b.clip (overwritten every iteration)
    k_transform_plain<<<dim3((p.n_verts + 255) / 256, p.views), 256, 0, s>>>(
            target_pos, b.mvps, p.n_verts, reinterpret_cast<float4*>(b.clip));
    hard_raster_op(hd, mem, b.clip, nullptr, b.faces, b.targets, nullptr,
                   b.soft.status, s);
    const size_t n = size_t(p.views) * p.res * p.res;
    k_mask_from_id<<<int(std::min<size_t>((n + 255) / 256, 8192)), 256, 0, s>>>(
            b.targets, n);
    check_launch();
    DRESSI_CUDA(cudaFreeAsync(mem, s));
    (void)d;
}

}  // namespace dressi
