// Test program: the silhouette optimisation (config C3) written against the
// C++ graph API (dressi/dressi.h), as a reference user writes it
// (examples/silhouette_optimization/run.cpp:228-437 of the reference):
// per view RasterizeSoft(SoftClip(clip)), pred = max(hard, soft), loss =
// SumPixelWise over views of (target - pred)^2 / R^2, the example's
// regulariser, in-graph Adam with addUpdate state, DressiAD::execStep.
//
//   graph_silhouette <in.bin> <out.bin>
// in.bin (little-endian): u32 n_verts, n_faces, n_views, res, n_iters,
//   max_deg_vf, max_deg_vn; f32 radius, sigma, lr, laplacian, normal;
//   f32 pos[V*3], faces[F*3], mvps[views*16], targets[views*R*R],
//   vft[max_deg_vf*V], vnb[max_deg_vn*V], fadj[F*3]
// out.bin: f32 loss_trace[n_iters], pos[V*3]
#include <cstdio>
#include <cstring>
#include <vector>

#include "dressi/dressi_ad.h"
#include "dressi/f.h"

using namespace dressi;

namespace {

template <typename T>
T read1(FILE* fp) {
    T v{};
    if (std::fread(&v, sizeof(T), 1, fp) != 1) throw DressiError("short read");
    return v;
}

std::vector<float> readn(FILE* fp, size_t n) {
    std::vector<float> v(n);
    if (n && std::fread(v.data(), 4, n, fp) != n)
        throw DressiError("short read");
    return v;
}

Variable ClipOf(const Variable& pos, const float* m) {
    Variable x = F::GetX(pos), y = F::GetY(pos), z = F::GetZ(pos);
    auto row = [&](int r) {
        return x * m[r] + y * m[4 + r] + z * m[8 + r] + m[12 + r];
    };
    return F::Vec4(row(0), row(1), row(2), row(3));
}

}  // namespace

int main(int argc, char** argv) {
    if (argc != 3) {
        std::fprintf(stderr, "usage: %s in.bin out.bin\n", argv[0]);
        return 2;
    }
    try {
        FILE* fi = std::fopen(argv[1], "rb");
        if (!fi) throw DressiError("cannot open input");
        const uint32_t nv = read1<uint32_t>(fi), nf = read1<uint32_t>(fi);
        const uint32_t views = read1<uint32_t>(fi), res = read1<uint32_t>(fi);
        const uint32_t iters = read1<uint32_t>(fi);
        const uint32_t deg_vf = read1<uint32_t>(fi);
        const uint32_t deg_vn = read1<uint32_t>(fi);
        const float radius = read1<float>(fi), sigma = read1<float>(fi);
        const float lr = read1<float>(fi), lap = read1<float>(fi);
        const float nrm = read1<float>(fi);
        const auto pos0 = readn(fi, size_t(nv) * 3);
        const auto faces = readn(fi, size_t(nf) * 3);
        const auto mvps = readn(fi, size_t(views) * 16);
        const auto targets = readn(fi, size_t(views) * res * res);
        const auto vft = readn(fi, size_t(deg_vf) * nv);
        const auto vnb = readn(fi, size_t(deg_vn) * nv);
        const auto fadj = readn(fi, size_t(nf) * 3);
        std::fclose(fi);

        const ImgSize screen{res, res};
        Variable pos(VEC3, {nv, 1}), faces_tex(VEC3, {nf, 1});
        Variable vft_tex(FLOAT, {nv, deg_vf}), face_id(FLOAT, {nf * 3, 1});
        Variable faces_soft(IVEC3, {nf, 1});
        Variables tgts, losses;
        const float k = (2.f / float(res)) * (2.f / float(res)) / sigma;
        for (uint32_t v = 0; v < views; v++) {
            tgts.emplace_back(FLOAT, screen);
            Variable clip = ClipOf(pos, mvps.data() + v * 16);
            Variable soft = F::SoftClip(clip, faces_tex, screen, radius);
            Variable rs = F::RasterizeSoft(soft, face_id, faces_soft, clip,
                                           faces_tex, vft_tex, screen, radius);
            Variable dist = F::GetX(rs), cov = F::GetW(rs);
            Variable hard = cov * F::Step(F::Float(0.f), dist);
            Variable sft = cov * F::Sigmoid(dist * F::Abs(dist) * k);
            Variable pred = F::Max(hard, sft);
            Variable diff = F::StopGradient(tgts.back()) - pred;
            losses.push_back(diff * diff * (1.f / float(res * res)));
        }
        Variable loss = F::SumPixelWise(losses);
        pos.setRequiresGradRecursively();

        DressiAD ad(0);
        ad.setLossVar(loss);
        Variable vnb_tex(FLOAT, {nv, deg_vn}), fadj_tex(VEC3, {nf, 1});
        ad.setOptimizer([&](Variables xs, Variables gxs) {
            Variables outs;
            for (size_t i = 0; i < xs.size(); i++) {
                Variable x = xs[i], g = gxs[i];
                if (lap != 0.f || nrm != 0.f) {
                    const float inv_cnt = 1.f / float(nv * 3);
                    auto rms = [&](const Variable& a) {
                        return F::Sqrt(F::SumAll(a * a) * inv_cnt + 1e-24f);
                    };
                    Variable data_rms = rms(g);
                    Variable g_lap = x - F::VertexNeighborMean(x, vnb_tex);
                    Variable g_nrm = F::NormalConsistencyVertexGrad(
                            F::NormalConsistencyFaceTerm(x, faces_tex,
                                                         fadj_tex),
                            x, faces_tex, vft_tex);
                    g = g + g_lap * (data_rms / rms(g_lap) * lap) +
                        g_nrm * (data_rms / rms(g_nrm) * nrm);
                }
                Variable m(VEC3, {nv, 1}), vv(VEC3, {nv, 1}), t(FLOAT, {1, 1});
                const float b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
                Variable t_new = t + 1.f;
                Variable m_new = m * b1 + g * (1.f - b1);
                Variable v_new = vv * b2 + g * g * (1.f - b2);
                Variable bc1 = 1.f - F::Pow(F::Float(b1), t_new);
                Variable bc2 = 1.f - F::Pow(F::Float(b2), t_new);
                Variable step =
                        (m_new / bc1) / (F::Sqrt(v_new / bc2) + eps) * lr;
                ad.addUpdate(m, m_new);
                ad.addUpdate(vv, v_new);
                ad.addUpdate(t, t_new);
                outs.push_back(x - step);
            }
            return outs;
        });
        std::vector<float> fid(size_t(nf) * 3), fsoft(size_t(nf) * 3);
        for (uint32_t f = 0; f < nf; f++)
            for (uint32_t c = 0; c < 3; c++) {
                fid[f * 3 + c] = float(f);
                fsoft[f * 3 + c] = float(f * 3 + c);
            }
        ad.sendImg(pos, CpuImageView(pos0.data(), nv, 1, 3));
        ad.sendImg(faces_tex, CpuImageView(faces.data(), nf, 1, 3));
        ad.sendImg(vft_tex, CpuImageView(vft.data(), nv, deg_vf, 1));
        ad.sendImg(vnb_tex, CpuImageView(vnb.data(), nv, deg_vn, 1));
        ad.sendImg(fadj_tex, CpuImageView(fadj.data(), nf, 1, 3));
        ad.sendImg(face_id, CpuImageView(fid.data(), nf * 3, 1, 1));
        ad.sendImg(faces_soft, CpuImageView(fsoft.data(), nf, 1, 3));
        for (uint32_t v = 0; v < views; v++)
            ad.sendImg(tgts[v], CpuImageView(targets.data() +
                                                     size_t(v) * res * res,
                                             res, res, 1));
        std::vector<float> trace;
        for (uint32_t it = 0; it < iters; it++) {
            ad.execStep();
            const CpuImage li = ad.recvImg(loss);
            double s = 0.0;
            for (float x : li.data) s += x;
            trace.push_back(float(s));
        }
        const CpuImage p = ad.recvImg(pos);
        if (ad.status() != 0) throw DressiError("device status word set");
        FILE* fo = std::fopen(argv[2], "wb");
        if (!fo) throw DressiError("cannot open output");
        std::fwrite(trace.data(), 4, trace.size(), fo);
        std::fwrite(p.data.data(), 4, p.data.size(), fo);
        std::fclose(fo);
        const auto st = ad.stats();
        std::printf("funcs %u exec %u steps %u programs %u kernels %u\n",
                    st.n_funcs, st.n_exec_funcs, st.n_steps, st.n_programs,
                    st.kernels_per_iter);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
    return 0;
}
