// Sparse GQA attention over an NVFP4 KV cache (the Qwen4-exp QSA / MiniMax sparse-decode shape: few KV heads, head
// dim up to 256, each query attending to its indexer's top-k cache slots), sm_100a.
//
//   qsa_kv_write   K or V rows [T, Hkv, D] BF16 -> NVFP4 cache rows of the given slots: codes [slots, Hkv, D/2] (E2M1,
//                  low nibble first) and one E4M3 scale per 16 values [slots, Hkv, D/16] (scale = amax / 6, no global
//                  scale: KV values are O(1)). One warp per (token, head), one lane per 16-value block.
//   qsa_partial    grid (key splits of 32, Hkv, B): the G = Hq / Hkv query heads of a KV head share every key and
//                  value the CTA dequantizes (the split's NVFP4 rows staged in shared memory in one round of 16-byte
//                  loads, decoded in registers, never stored as BF16). Scores: a
//                  warp per key, each lane D/32 values of the row, all G heads' dots reduced with shuffles; softmax
//                  of the split per head (max, exponentials, sum); P.V: a thread per value dimension, G accumulators.
//                  Writes the split's unnormalized output and (max, sum) per head.
//   qsa_merge      grid (Hq, B): the splits of a head combined by their maxima (the log-sum-exp merge of split-K
//                  decoding) into BF16; a head with no valid key gets zeros.
// Key slots of -1 (fewer selected keys than nsel) are skipped. Decode is bound by the gathered cache bytes
// (D * 5/8 + ... per key and head for K and V together), so the work stays on CUDA cores like the other decode
// attention paths.
#include <cuda_runtime.h>

#include "common.cuh"

namespace xt {

constexpr int QSA_KEYS = 32, QSA_THREADS = 256, QSA_MAX_G = 16, QSA_MAX_D = 256, QSA_MAX_SPLITS = 1024;
#define QSA_NEG_INF __int_as_float(0xff800000)

__global__ void __launch_bounds__(256) qsa_kv_write_kernel(const __nv_bfloat16 *__restrict__ x,
                                                           const int64_t *__restrict__ slot, uint8_t *codes,
                                                           uint8_t *scales, int T, int H, int D) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= T * H || lane >= D / 16) return;
    const int t = row / H, h = row % H;
    const size_t dst = size_t(slot[t]) * H + h;
    const uint4 *src = reinterpret_cast<const uint4 *>(x + size_t(row) * D + lane * 16);
    float v[16];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const uint4 u = src[c];
        const __nv_bfloat162 *b = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(b[i]);
            v[c * 8 + 2 * i] = f.x;
            v[c * 8 + 2 * i + 1] = f.y;
        }
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const uint8_t sc = f32_to_e4m3(amax / 6.f);
    const float sf = e4m3_to_f(sc);
    const float inv = sf > 0.f ? 1.f / sf : 0.f;
    uint32_t w[2];
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t acc = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            acc |= uint32_t(f32x2_to_e2m1(v[h2 * 8 + 2 * i] * inv, v[h2 * 8 + 2 * i + 1] * inv)) << (8 * i);
        w[h2] = acc;
    }
    *reinterpret_cast<uint2 *>(codes + dst * (D / 2) + lane * 8) = make_uint2(w[0], w[1]);
    scales[dst * (D / 16) + lane] = sc;
}

// E2M1 code -> value (the format's eight magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6; sign in bit 3)
XT_DEV float e2m1_val(uint32_t c) {
    const float a = (c & 4) ? ((c & 2) ? ((c & 1) ? 6.f : 4.f) : ((c & 1) ? 3.f : 2.f))
                            : ((c & 2) ? ((c & 1) ? 1.5f : 1.f) : ((c & 1) ? 0.5f : 0.f));
    return (c & 8) ? -a : a;
}

struct QsaParams {
    const __nv_bfloat16 *q;   // [B, Hq, D]
    const int32_t *idx;       // [B, nsel] cache slots, -1 = none
    const uint8_t *kc, *ks, *vc, *vs;   // [slots, Hkv, D/2], [slots, Hkv, D/16]
    float *part_o;            // [B, Hkv, splits, G, D]
    float *part_ml;           // [B, Hkv, splits, G, 2]
    __nv_bfloat16 *out;       // [B, Hq, D]
    int B, nsel, Hq, Hkv, G, D, splits;
    float scale;
};

// The split's keys and values are brought into shared memory first (every 16-byte piece of the 32 rows' codes and
// scales requested at once: one memory round trip), then decoded from there.
__global__ void __launch_bounds__(QSA_THREADS) qsa_partial_kernel(QsaParams p) {
    constexpr int CB = QSA_MAX_D / 2, SB = QSA_MAX_D / 16;   // row bytes of codes / scales at the largest D
    __shared__ float qs[QSA_MAX_G * QSA_MAX_D];
    __shared__ float sc[QSA_MAX_G * QSA_KEYS];
    __shared__ __align__(16) uint8_t kcs[QSA_KEYS * CB], vcs[QSA_KEYS * CB];
    __shared__ __align__(16) uint8_t kss[QSA_KEYS * SB], vss[QSA_KEYS * SB];
    __shared__ int slots[QSA_KEYS];
    __shared__ float ml[QSA_MAX_G * 2];
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = p.G, D = p.D, cb = D / 2, sb = D / 16;
    if (tid < QSA_KEYS) {
        const int j = split * QSA_KEYS + tid;
        slots[tid] = j < p.nsel ? p.idx[size_t(b) * p.nsel + j] : -1;
    }
    // queries in lane-major order (element d = lane * D/32 + e at g * D + e * 32 + lane): the score loop's reads
    // are then conflict-free across the warp
    for (int i = tid; i < G * D; i += QSA_THREADS) {
        const int g = i / D, d = i % D, epl_ = D / 32;
        qs[g * D + (d % epl_) * 32 + d / epl_] =
            __bfloat162float(p.q[(size_t(b) * p.Hq + size_t(kvh) * G + g) * D + d]);
    }
    __syncthreads();
    {   // codes: cb / 16 pieces per row; scales: one piece per row (sb <= 16) -- K and V
        const int cp = cb / 16, n_code = QSA_KEYS * cp;
        for (int i = tid; i < 2 * n_code + 2 * QSA_KEYS; i += QSA_THREADS) {
            const bool val = i >= n_code + QSA_KEYS;
            const int k = val ? i - n_code - QSA_KEYS : i;
            const int key = k < n_code ? k / cp : k - n_code;
            const int s = slots[key];
            if (s < 0) continue;
            const size_t r = size_t(s) * p.Hkv + kvh;
            if (k < n_code) {
                const int c = k % cp;
                const uint4 v = *reinterpret_cast<const uint4 *>((val ? p.vc : p.kc) + r * cb + c * 16);
                *reinterpret_cast<uint4 *>((val ? vcs : kcs) + key * CB + c * 16) = v;
            } else {   // one load of the row's sb scale bytes (sb = D/16: 2, 4, 8 or 16, aligned to its size)
                const uint8_t *src = (val ? p.vs : p.ks) + r * sb;
                uint8_t *dst = (val ? vss : kss) + key * SB;
                if (sb == 16) *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(src);
                else if (sb == 8) *reinterpret_cast<uint2 *>(dst) = *reinterpret_cast<const uint2 *>(src);
                else if (sb == 4) *reinterpret_cast<uint32_t *>(dst) = *reinterpret_cast<const uint32_t *>(src);
                else *reinterpret_cast<uint16_t *>(dst) = *reinterpret_cast<const uint16_t *>(src);
            }
        }
    }
    __syncthreads();
    // scores: a warp per key; lane covers D/32 consecutive values (inside one 16-value scale block)
    const int epl = D / 32, d0 = lane * epl;
    for (int jj = warp; jj < QSA_KEYS; jj += QSA_THREADS / 32) {
        if (slots[jj] < 0) {
            if (lane < G) sc[lane * QSA_KEYS + jj] = QSA_NEG_INF;
            continue;
        }
        const uint8_t *kc = kcs + jj * CB;
        const float ksf = e4m3_to_f(kss[jj * SB + d0 / 16]);
        float k[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            if (e < epl) {
                const int d = d0 + e;
                const uint32_t byte = kc[d / 2];
                k[e] = e2m1_val((d & 1) ? byte >> 4 : byte & 15) * ksf;
            }
        }
        for (int g = 0; g < G; ++g) {
            float acc = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e)
                if (e < epl) acc += qs[g * D + e * 32 + lane] * k[e];
#pragma unroll
            for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (lane == 0) sc[g * QSA_KEYS + jj] = acc * p.scale;
        }
    }
    __syncthreads();
    // softmax of the split, per head: a warp per head, one key per lane
    for (int g = warp; g < G; g += QSA_THREADS / 32) {
        const float s0 = sc[g * QSA_KEYS + lane];
        float m = s0;
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float p0 = m == QSA_NEG_INF ? 0.f : __expf(s0 - m);
        float l = p0;
#pragma unroll
        for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        sc[g * QSA_KEYS + lane] = p0;
        if (lane == 0) {
            ml[2 * g] = m;
            ml[2 * g + 1] = l;
        }
    }
    __syncthreads();
    // P.V: a thread per value dimension, all heads of the group
    const size_t base = (size_t(b) * p.Hkv + kvh) * p.splits + split;
    for (int d = tid; d < D; d += QSA_THREADS) {
        float acc[QSA_MAX_G];
#pragma unroll
        for (int g = 0; g < QSA_MAX_G; ++g) acc[g] = 0.f;
        for (int jj = 0; jj < QSA_KEYS; ++jj) {
            if (slots[jj] < 0) continue;
            const uint32_t byte = vcs[jj * CB + d / 2];
            const float v = e2m1_val((d & 1) ? byte >> 4 : byte & 15) * e4m3_to_f(vss[jj * SB + d / 16]);
#pragma unroll
            for (int g = 0; g < QSA_MAX_G; ++g)
                if (g < G) acc[g] += sc[g * QSA_KEYS + jj] * v;
        }
#pragma unroll
        for (int g = 0; g < QSA_MAX_G; ++g)
            if (g < G) p.part_o[(base * G + g) * D + d] = acc[g];
    }
    if (tid < 2 * G) p.part_ml[base * G * 2 + tid] = ml[tid];
}

// The split weights exp(m_s - M) / L are computed once per head by warp 0 into shared memory; the value loop then
// issues independent loads of the splits' partial outputs.
__global__ void __launch_bounds__(QSA_THREADS) qsa_merge_kernel(QsaParams p) {
    __shared__ float wsp[QSA_MAX_SPLITS];
    const int hq = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
    const int kvh = hq / p.G, g = hq % p.G, D = p.D, S = p.splits;
    const size_t base = (size_t(b) * p.Hkv + kvh) * S;
    if (tid < 32) {
        float M = QSA_NEG_INF;
        for (int s = lane; s < S; s += 32) M = fmaxf(M, p.part_ml[((base + s) * p.G + g) * 2]);
#pragma unroll
        for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float L = 0.f;
        for (int s = lane; s < S; s += 32) {
            const float m = p.part_ml[((base + s) * p.G + g) * 2];
            const float e = m == QSA_NEG_INF ? 0.f : __expf(m - M);
            wsp[s] = e;
            L += e * p.part_ml[((base + s) * p.G + g) * 2 + 1];
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        const float inv = L > 0.f ? 1.f / L : 0.f;
        for (int s = lane; s < S; s += 32) wsp[s] *= inv;
    }
    __syncthreads();
    for (int d = tid; d < D; d += QSA_THREADS) {
        float o = 0.f;
#pragma unroll 4
        for (int s = 0; s < S; ++s) o += wsp[s] * p.part_o[((base + s) * p.G + g) * D + d];
        p.out[(size_t(b) * p.Hq + hq) * D + d] = __float2bfloat16(o);
    }
}

}  // namespace xt

extern "C" int xt_qsa_kv_write(const void *x, const int64_t *slot, int T, int H, int D, void *codes, void *scales,
                               cudaStream_t stream) {
    if (T <= 0 || H <= 0 || D % 32 || D < 32 || D > 512) return -2;
    const int warps = 8, rows = T * H;
    xt::qsa_kv_write_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, stream>>>(
        static_cast<const __nv_bfloat16 *>(x), slot, static_cast<uint8_t *>(codes), static_cast<uint8_t *>(scales), T,
        H, D);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// Attention of B decode queries (Hq heads of dim D) over their selected cache slots: out [B, Hq, D] BF16 =
// softmax(scale * q.k) . v, keys and values dequantized from the NVFP4 cache. Scratch: part_o [B, Hkv, splits, G, D]
// and part_ml [B, Hkv, splits, G, 2] FP32 with splits = ceil(nsel / 32).
extern "C" int xt_qsa_decode(const void *q, const int32_t *idx, int B, int nsel, int Hq, int Hkv, int D,
                             const void *kc, const void *ks, const void *vc, const void *vs, float *part_o,
                             float *part_ml, void *out, float scale, cudaStream_t stream) {
    if (B <= 0 || nsel <= 0 || Hkv <= 0 || Hq % Hkv || D % 32 || D < 32 || D > xt::QSA_MAX_D) return -2;
    if ((nsel + xt::QSA_KEYS - 1) / xt::QSA_KEYS > xt::QSA_MAX_SPLITS) return -2;   // nsel <= 32768
    const int G = Hq / Hkv;
    if (G > xt::QSA_MAX_G) return -2;
    xt::QsaParams p{};
    p.q = static_cast<const __nv_bfloat16 *>(q);
    p.idx = idx;
    p.kc = static_cast<const uint8_t *>(kc);
    p.ks = static_cast<const uint8_t *>(ks);
    p.vc = static_cast<const uint8_t *>(vc);
    p.vs = static_cast<const uint8_t *>(vs);
    p.part_o = part_o;
    p.part_ml = part_ml;
    p.out = static_cast<__nv_bfloat16 *>(out);
    p.B = B;
    p.nsel = nsel;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.G = G;
    p.D = D;
    p.splits = (nsel + xt::QSA_KEYS - 1) / xt::QSA_KEYS;   // (part_o / part_ml sized for 32-key splits)
    p.scale = scale;
    xt::qsa_partial_kernel<<<dim3(p.splits, Hkv, B), xt::QSA_THREADS, 0, stream>>>(p);
    if (cudaGetLastError() != cudaSuccess) return -1;
    xt::qsa_merge_kernel<<<dim3(Hq, B), xt::QSA_THREADS, 0, stream>>>(p);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
