// Kernel selection and launch for the SIMT strided GEMM (gemm_simt.cuh).
#include <algorithm>

#include "gemm_simt.cuh"
#include "kx_internal.hpp"

namespace kx {

namespace {

// 128x128 tiles, 8x8 outputs per thread, 256 threads (two CTAs per SM for f32).
template <typename T> struct BigCfg;
template <> struct BigCfg<float> : TileCfg<float, 128, 128, KX_F32_BK, 8, 8, KX_F32_MINB> {};
template <> struct BigCfg<double> : TileCfg<double, 128, 128, 8, 8, 8, 1> {};
// 64x64 tiles, 4x4 per thread: more CTAs for small or split-K problems.
template <typename T> struct SmallCfg;
template <> struct SmallCfg<float> : TileCfg<float, 64, 64, 16, 4, 4, 2> {};
template <> struct SmallCfg<double> : TileCfg<double, 64, 64, 16, 4, 4, 2> {};

template <typename T, typename Cfg, int AM, int BMD, bool ORD>
cudaError_t launch_one(const GemmParams<T> &p, cudaStream_t s) {
    const int64_t tiles = (int64_t)((p.M + Cfg::BM - 1) / Cfg::BM) * ((p.N + Cfg::BN - 1) / Cfg::BN);
    const int64_t z = p.nbatch * p.splits;
    dim3 grid((unsigned)tiles, (unsigned)(z < 65535 ? z : 65535), 1);
    gemm_simt_kernel<T, Cfg, AM, BMD, ORD><<<grid, Cfg::NT, 0, s>>>(p);
    return cudaGetLastError();
}

template <typename T, typename Cfg, int AM, bool ORD>
cudaError_t launch_b(const GemmParams<T> &p, int bmode, cudaStream_t s) {
    switch (bmode) {
        case kVecK: return launch_one<T, Cfg, AM, kVecK, ORD>(p, s);
        case kVecMN: return launch_one<T, Cfg, AM, kVecMN, ORD>(p, s);
        case kGatherMN: return launch_one<T, Cfg, AM, kGatherMN, ORD>(p, s);
        default: return launch_one<T, Cfg, AM, kGatherK, ORD>(p, s);
    }
}

template <typename T, typename Cfg, bool ORD = false>
cudaError_t launch_cfg(const GemmParams<T> &p, int amode, int bmode, cudaStream_t s) {
    switch (amode) {
        case kVecK: return launch_b<T, Cfg, kVecK, ORD>(p, bmode, s);
        case kVecMN: return launch_b<T, Cfg, kVecMN, ORD>(p, bmode, s);
        case kGatherMN: return launch_b<T, Cfg, kGatherMN, ORD>(p, bmode, s);
        default: return launch_b<T, Cfg, kGatherK, ORD>(p, bmode, s);
    }
}

inline int64_t iabs(int64_t v) { return v < 0 ? -v : v; }

// Operand access mode.  `s_r` is the stride along m (A) or n (B), `s_k` along k,
// `R` the extent along m/n.  `batch_ok` says every batch stride and the origin
// keep vector alignment.
template <typename T>
int pick_mode(const T *base, int64_t s_r, int64_t s_k, int64_t R, int64_t K, bool batch_ok) {
    constexpr int W = Vec<T>::width;
    const bool aligned = batch_ok && (reinterpret_cast<uintptr_t>(base) % (W * sizeof(T)) == 0);
    if (aligned && s_k == 1 && K % W == 0 && s_r % W == 0) return kVecK;
    if (aligned && s_r == 1 && R % W == 0 && s_k % W == 0) return kVecMN;
    return iabs(s_r) <= iabs(s_k) ? kGatherMN : kGatherK;
}

}  // namespace

template <typename T>
int run_gemm(Handle *h, GemmParams<T> p, const char **kernel_name) {
    constexpr int W = Vec<T>::width;
    bool a_batch_ok = true, b_batch_ok = true;
    for (int d = 0; d < p.batch.ndims; ++d) {
        a_batch_ok &= (p.batch.a_str[d] % W) == 0;
        b_batch_ok &= (p.batch.b_str[d] % W) == 0;
    }
    const int amode = pick_mode<T>(p.A, p.a_rs, p.a_cs, p.M, p.K, a_batch_ok);
    const int bmode = pick_mode<T>(p.B, p.b_cs, p.b_rs, p.N, p.K, b_batch_ok);

    using Big = BigCfg<T>;
    using Small = SmallCfg<T>;
    const int64_t target = 2LL * h->sm_count;  // two resident CTAs per SM
    const int64_t big_tiles = (int64_t)((p.M + Big::BM - 1) / Big::BM) * ((p.N + Big::BN - 1) / Big::BN);
    const int64_t small_tiles = (int64_t)((p.M + Small::BM - 1) / Small::BM) * ((p.N + Small::BN - 1) / Small::BN);
    if (big_tiles > INT32_MAX || small_tiles > INT32_MAX) return KX_E_UNSUPPORTED;

    p.splits = 1;
    p.k_per_split = p.K;
    p.ws = nullptr;
    cudaError_t ce;
    if constexpr (std::is_same<T, float>::value) {
        // Split-TF32 tensor-core path: eligible layouts, enough 128x256 tiles to
        // fill the machine, and not the ordered (bitwise reference) mode.
        if (!h->ordered && h->f32_variant != KX_F32_FFMA && tc_eligible(p)) {
            const int64_t sms = h->sm_count;
            const int64_t tc_tiles = (int64_t)((p.M + 127) / 128) * ((p.N + 255) / 256) * p.nbatch;
            const bool big = tc_tiles >= sms / 2 && p.K >= 64;
            if (h->f32_variant == KX_F32_3XTF32 || h->f32_variant == KX_F32_3XTF32_1SM || big) {
                // CTA pairs or one-SM tiles by the wave model: waves of
                // sm_count CTAs times a per-CTA cost of (width + 32), a
                // 256-wide pair CTA (128 rows x 256) running ~8 % faster for
                // the lighter shared-memory traffic (measured: 222 vs 205
                // TFLOP/s at 8192^3; the 224-wide pair, which stages 128 B
                // columns for 112, is slower than one-SM 224-wide tiles);
                // pairs only for K long enough to amortise their cluster set-up.
                auto waves = [&](int64_t ctas) { return (ctas + sms - 1) / sms; };
                const int64_t tm1 = (p.M + 127) / 128, tmp = (p.M + 255) / 256;
                double best1 = 1e30, bestp = 1e30;
                for (int bn : {256, 224, 128})
                    best1 = std::min(best1, (double)waves(tm1 * ((p.N + bn - 1) / bn) * p.nbatch) * (bn + 32));
                bestp = 0.92 * (double)waves(2 * tmp * ((p.N + 255) / 256) * p.nbatch) * (256 + 32);
                int rc = KX_DECLINED;
                // Short contractions over many tiles: the persistent kernel,
                // whose epilogue overlaps the next tile.
                const int64_t tiles128 = tm1 * ((p.N + 127) / 128) * p.nbatch;
                if (h->f32_variant == KX_F32_AUTO && !p.C_mc && p.K <= 1024 && tiles128 >= 2LL * sms)
                    rc = run_gemm_tc_short(h, p, kernel_name);
                if (rc == KX_DECLINED && h->f32_variant != KX_F32_3XTF32_1SM && !p.C_mc && p.M >= 256 &&
                    (h->f32_variant == KX_F32_3XTF32 || (p.K >= 512 && bestp < best1)))
                    rc = run_gemm_tc_pair(h, p, kernel_name);
                if (rc == KX_DECLINED) rc = run_gemm_tc(h, p, kernel_name);   // one-SM tiles
                if (rc != KX_DECLINED) return rc;
            } else if (h->f32_variant == KX_F32_AUTO && p.nbatch == 1 && !p.C_mc && p.K >= 256) {
                // Too few tiles to fill the SMs: split K over the tensor-core
                // kernel, describing the K slices as a batch (A's batch stride
                // the slice width, B's that many rows, the partial products in
                // the workspace) and summing the slices in increasing order.
                // A single tile over a long K is latency-bound on one SM
                // (about 4x its MMA time); slices of >= 64 k spread it out.
                const int64_t tiles = ((p.M + 127) / 128) * ((p.N + 127) / 128);
                int splits = 1;
                while (tiles * splits * 2 <= sms && p.K % (int64_t)(splits * 2 * 16) == 0 &&
                       p.K / (splits * 2) >= 64)
                    splits *= 2;
                // (a CTA's few microseconds of latency against 10-20 us for the
                // SIMT split-K kernel on such shapes, measured: worth it from 32 CTAs)
                if (splits >= 2 && tiles * splits >= 32) {
                    const int kps = p.K / splits;
                    const uint64_t need = (uint64_t)splits * p.M * p.N * sizeof(float);
                    float *ws = nullptr;
                    int rc = h->workspace(need, reinterpret_cast<void **>(&ws));
                    if (rc) return rc;
                    GemmParams<T> q = p;
                    q.K = kps;
                    q.C = ws;
                    q.c_rs = p.N;
                    q.c_cs = 1;
                    q.nbatch = splits;
                    q.batch.ndims = 1;
                    q.batch.dims[0] = splits;
                    q.batch.a_str[0] = (int64_t)kps * p.a_cs;
                    q.batch.b_str[0] = (int64_t)kps * p.b_rs;
                    q.batch.c_str[0] = (int64_t)p.M * p.N;
                    if (tc_eligible(q)) {
                        rc = run_gemm_tc(h, q, kernel_name);
                        if (rc == KX_OK) {
                            GemmParams<T> r = p;
                            r.ws = ws;
                            r.splits = splits;
                            const int64_t total = (int64_t)p.M * p.N;
                            int64_t blocks = (total + 255) / 256;
                            if (blocks > 8LL * h->sm_count) blocks = 8LL * h->sm_count;
                            splitk_reduce_kernel<T><<<(unsigned)blocks, 256, 0, h->stream>>>(r);
                            ++h->launches;
                            ce = cudaGetLastError();
                            if (ce != cudaSuccess) return h->cuda_fail(ce);
                            *kernel_name = "tc_3xtf32_splitk";
                            return KX_OK;
                        }
                        if (rc != KX_DECLINED) return rc;
                    }
                }
            }
        }
    }
    if constexpr (std::is_same<T, double>::value) {
        // FP64 tensor pipe for layouts with a unit stride along k or m/n and
        // enough 128x128 tiles to spread over the SMs.
        if (!h->ordered && h->f64_variant != KX_F64_DFMA) {
            const int64_t tiles = (int64_t)((p.M + 127) / 128) * ((p.N + 127) / 128) * p.nbatch;
            if (h->f64_variant == KX_F64_DMMA || tiles >= h->sm_count / 2) {
                int rc = run_gemm_dmma(h, p, kernel_name);
                if (rc == KX_OK && p.C_mc) return mc_copy(h, p.C, p.C_mc, (uint64_t)p.nbatch * p.M * p.N * sizeof(T));
                if (rc != KX_DECLINED) return rc;
            }
        }
    }
    if (h->ordered) {
        // Ordered mode: one pass over k per output, separately rounded
        // multiply and add -- bitwise equal to the reference's ordered path.
        *kernel_name = "simt_64x64_ordered";
        ce = launch_cfg<T, Small, true>(p, amode, bmode, h->stream);
        ++h->launches;
    } else if (big_tiles * p.nbatch >= target) {
        *kernel_name = "simt_128x128";
        ce = launch_cfg<T, Big>(p, amode, bmode, h->stream);
        ++h->launches;
    } else {
        // Split K so that the grid fills the machine; each split keeps at least
        // four k-tiles so the pipeline stays primed.
        int64_t ctas = small_tiles * p.nbatch;
        int splits = 1;
        if (ctas < target) {
            int64_t want = (target + ctas - 1) / ctas;
            int64_t max_splits = p.K / (4 * Small::BK);
            if (max_splits < 1) max_splits = 1;
            splits = (int)(want < max_splits ? want : max_splits);
        }
        if (splits > 1) {
            int64_t kps = (p.K + splits - 1) / splits;
            kps = (kps + Small::BK - 1) / Small::BK * Small::BK;
            splits = (int)((p.K + kps - 1) / kps);
            p.k_per_split = (int)kps;
        }
        p.splits = splits;
        if (splits > 1) {
            const uint64_t need = (uint64_t)splits * p.nbatch * (uint64_t)p.M * p.N * sizeof(T);
            int rc = h->workspace(need, reinterpret_cast<void **>(&p.ws));
            if (rc) return rc;
            *kernel_name = "simt_64x64_splitk";
        } else {
            *kernel_name = "simt_64x64";
        }
        ce = launch_cfg<T, Small>(p, amode, bmode, h->stream);
        ++h->launches;
        if (ce == cudaSuccess && splits > 1) {
            const int64_t total = p.nbatch * (int64_t)p.M * p.N;
            int64_t blocks = (total + 255) / 256;
            if (blocks > 8LL * h->sm_count) blocks = 8LL * h->sm_count;
            splitk_reduce_kernel<T><<<(unsigned)blocks, 256, 0, h->stream>>>(p);
            ce = cudaGetLastError();
            ++h->launches;
        }
    }
    if (ce == cudaSuccess && p.C_mc) {
        // The SIMT kernels store locally; the rows then go out through the
        // multicast address (C is C-contiguous here).
        return mc_copy(h, p.C, p.C_mc, (uint64_t)p.nbatch * p.M * p.N * sizeof(T));
    }
    return ce == cudaSuccess ? KX_OK : h->cuda_fail(ce);
}

template int run_gemm<float>(Handle *, GemmParams<float>, const char **);
template int run_gemm<double>(Handle *, GemmParams<double>, const char **);

}  // namespace kx
