// tb_dequant.cu — bit-exact dequantisation of GGUF rows to fp32 on sm_100a.
//
// One thread produces 8 consecutive weights of the flat M*K output.  Every
// product and difference is an explicit IEEE round-to-nearest operation
// (__fmul_rn / __fsub_rn) in the reference's evaluation order, so no FMA
// contraction can change a bit.  sem = 0 reproduces the reference CUDA kernels
// (layer4/tb_gguf_dequant.cu:89-332; Q2_K from layer4/tb_gguf.c:210-225);
// sem = 1 reproduces layer4/tb_gguf.c's shipped scale unpack for Q4_K
// (tb_gguf.c:163-168) and Q5_K (tb_gguf.c:130-144, via :270).
#include "tb_common.cuh"
#include "tb_internal.h"

namespace tb {

__device__ __forceinline__ uint32_t b8(const uint8_t *p, int i) { return __ldg(p + i); }
__device__ __forceinline__ uint32_t b16(const uint8_t *p, int i) { return b8(p, i) | (b8(p, i + 1) << 8); }

// 6-bit scale s and min m of sub-block j for Q4_K/Q5_K.
template <int QT, int SEM>
__device__ __forceinline__ void sm6(const uint8_t *sc, int j, uint32_t &s, uint32_t &m)
{
    if (SEM == 1 && QT == QT_Q4_K) {           // tb_gguf.c:163-168
        s = b8(sc, j < 4 ? j : j + 4) & 63u;
        m = b8(sc, j < 4 ? j + 4 : j + 8) & 63u;
    } else if (j < 4) {                          // tb_gguf_dequant.cu:104-105
        s = b8(sc, j) & 63u;
        m = b8(sc, j + 4) & 63u;
    } else {
        const int k = j - 4;
        s = (b8(sc, k) >> 6) | ((b8(sc, k + 8) & 15u) << 2);        // :106
        if (SEM == 1)                                              // tb_gguf.c:139
            m = (b8(sc, k + 4) >> 6) | ((b8(sc, k + 12) & 15u) << 2);
        else                                                       // :107
            m = (b8(sc, k + 4) >> 6) | ((b8(sc, k + 8) >> 4) << 2);
    }
}

// weight i of the block at b
template <int QT, int SEM>
__device__ __forceinline__ float deq1(const uint8_t *b, int i)
{
    if (QT == QT_F32) return __uint_as_float(b16(b, 4 * i) | (b16(b, 4 * i + 2) << 16));
    if (QT == QT_F16) return h2f_ref(b16(b, 2 * i));
    if (QT == QT_BF16) return bf2f(b16(b, 2 * i));
    if (QT == QT_Q4_0) {
        const float d = h2f_ref(b16(b, 0));
        const uint32_t q = (b8(b, 2 + (i >> 1)) >> ((i & 1) * 4)) & 15u;
        return __fmul_rn(d, static_cast<float>(static_cast<int>(q) - 8));
    }
    if (QT == QT_Q8_0) {
        const float d = h2f_ref(b16(b, 0));
        return __fmul_rn(d, static_cast<float>(static_cast<int8_t>(b8(b, 2 + i))));
    }
    if (QT == QT_Q8_K) {
        const float d = __uint_as_float(b16(b, 0) | (b16(b, 2) << 16));
        return __fmul_rn(d, static_cast<float>(static_cast<int8_t>(b8(b, 4 + i))));
    }
    if (QT == QT_Q2_K) {
        const float d = h2f_ref(b16(b, 80)), dmin = h2f_ref(b16(b, 82));
        const uint32_t sb = b8(b, i >> 4);
        const float sc = __fmul_rn(d, static_cast<float>(sb & 15u));
        const float mn = __fmul_rn(dmin, static_cast<float>(sb >> 4));
        const uint32_t q = (b8(b, 16 + (i >> 2)) >> ((i & 3) * 2)) & 3u;
        return __fsub_rn(__fmul_rn(sc, static_cast<float>(q)), mn);
    }
    if (QT == QT_Q3_K || QT == QT_IQ3_S) {
        const float d = h2f_ref(b16(b, 108));
        const int j = i >> 4, is = j < 8 ? j : j - 8;
        const uint32_t lo4 = (b8(b, 96 + (is >> 1)) >> ((is & 1) * 4)) & 15u;
        const uint32_t hi2 = (b8(b, 104 + (is >> 2)) >> ((is & 3) * 2)) & 3u;
        const float S = __fmul_rn(d, static_cast<float>(static_cast<int>(lo4 | (hi2 << 4)) - 32));
        const uint32_t l = (b8(b, 32 + (i >> 2)) >> ((i & 3) * 2)) & 3u;
        const uint32_t h = (b8(b, i >> 3) >> (i & 7)) & 1u;
        return __fmul_rn(S, static_cast<float>(static_cast<int>(l | (h << 2)) - 4));
    }
    if (QT == QT_Q4_K || QT == QT_Q5_K) {
        const float d = h2f_ref(b16(b, 0)), dmin = h2f_ref(b16(b, 2));
        uint32_t s, m;
        sm6<QT, SEM>(b + 4, i >> 5, s, m);
        const float S = __fmul_rn(d, static_cast<float>(s));
        const float Mn = __fmul_rn(dmin, static_cast<float>(m));
        uint32_t q;
        if (QT == QT_Q4_K) {
            q = (b8(b, 16 + (i >> 1)) >> ((i & 1) * 4)) & 15u;
        } else {
            const uint32_t lo = (b8(b, 48 + (i >> 1)) >> ((i & 1) * 4)) & 15u;
            const uint32_t hi = (b8(b, 16 + (i >> 3)) >> (i & 7)) & 1u;
            q = lo | (hi << 4);
        }
        return __fsub_rn(__fmul_rn(S, static_cast<float>(q)), Mn);
    }
    if (QT == QT_Q6_K) {
        const float d = h2f_ref(b16(b, 208));
        const int sc = static_cast<int8_t>(b8(b, 192 + (i >> 4)));
        const uint32_t lo = (b8(b, i >> 1) >> ((i & 1) * 4)) & 15u;
        const uint32_t hi = (b8(b, 128 + (i >> 2)) >> ((i & 3) * 2)) & 3u;
        return __fmul_rn(__fmul_rn(d, static_cast<float>(sc)),
                         static_cast<float>(static_cast<int>(lo | (hi << 4)) - 32));
    }
    return 0.f;
}

template <int QT, int SEM>
__global__ void __launch_bounds__(256) k_dequant(const uint8_t *__restrict__ W, uint32_t M,
                                                 uint32_t K, unsigned long long row_bytes,
                                                 float *__restrict__ out)
{
    constexpr Geom g = geom_of(QT);
    const unsigned long long total = static_cast<unsigned long long>(M) * K;
    const unsigned long long nchunk = (total + 7) / 8;
    for (unsigned long long c = blockIdx.x * 256ull + threadIdx.x; c < nchunk;
         c += static_cast<unsigned long long>(gridDim.x) * 256ull) {
        float v[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const unsigned long long e = c * 8 + t;
            v[t] = 0.f;
            if (e < total) {
                const uint32_t m = static_cast<uint32_t>(e / K), k = static_cast<uint32_t>(e % K);
                const uint8_t *blk = W + m * row_bytes +
                                     static_cast<unsigned long long>(k / g.block_weights) * g.block_bytes;
                v[t] = deq1<QT, SEM>(blk, static_cast<int>(k % g.block_weights));
            }
        }
        if (c * 8 + 8 <= total) {
            float4 *o = reinterpret_cast<float4 *>(out + c * 8);
            o[0] = make_float4(v[0], v[1], v[2], v[3]);
            o[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
            for (int t = 0; t < 8 && c * 8 + t < total; ++t) out[c * 8 + t] = v[t];
        }
    }
}

// One embedding row, selected on the device (the decode step's first kernel).
template <int QT>
__global__ void __launch_bounds__(256) k_embed_row(const uint8_t *__restrict__ W, uint32_t vocab, uint32_t K,
                                                   unsigned long long row_bytes, const int *token,
                                                   float *__restrict__ out)
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    constexpr Geom g = geom_of(QT);
    // grid.y > 1: a batch of tokens (token[y] into row y of out)
    const int t = token[blockIdx.y];
    out += static_cast<size_t>(blockIdx.y) * K;
    const bool ok = t >= 0 && static_cast<uint32_t>(t) < vocab;
    const uint8_t *row = W + (ok ? static_cast<unsigned long long>(t) * row_bytes : 0ull);
    for (uint32_t k = blockIdx.x * 256u + threadIdx.x; k < K; k += gridDim.x * 256u)
        out[k] = ok ? deq1<QT, 0>(row + static_cast<unsigned long long>(k / g.block_weights) * g.block_bytes,
                                  static_cast<int>(k % g.block_weights))
                    : 0.f;
}

template <int QT>
static int embed_go(const void *W, int vocab, int K, const int *tok, float *out, cudaStream_t st, int n = 1)
{
    constexpr Geom g = geom_of(QT);
    const unsigned long long row_bytes = static_cast<unsigned long long>(K / g.block_weights) * g.block_bytes;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>((K + 255) / 256), static_cast<unsigned>(n));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_embed_row<QT>, static_cast<const uint8_t *>(W), static_cast<uint32_t>(vocab),
                              static_cast<uint32_t>(K), row_bytes, tok, out) == cudaSuccess ? 1 : 0;
}

int dq_embed_launch(const void *W, int qtype, int vocab, int K, const int *d_token, float *d_out, cudaStream_t st,
                    int n)
{
    const Geom g = geom_of(qtype);
    if (!g.block_weights || !W || !d_token || !d_out || vocab <= 0 || K <= 0 || K % g.block_weights || n < 1 ||
        n > 65535)
        return 0;
    switch (qtype) {
    case QT_F32: return embed_go<QT_F32>(W, vocab, K, d_token, d_out, st, n);
    case QT_F16: return embed_go<QT_F16>(W, vocab, K, d_token, d_out, st, n);
    case QT_BF16: return embed_go<QT_BF16>(W, vocab, K, d_token, d_out, st, n);
    case QT_Q4_0: return embed_go<QT_Q4_0>(W, vocab, K, d_token, d_out, st, n);
    case QT_Q8_0: return embed_go<QT_Q8_0>(W, vocab, K, d_token, d_out, st, n);
    case QT_Q8_K: return embed_go<QT_Q8_K>(W, vocab, K, d_token, d_out, st, n);
    case QT_Q2_K: return embed_go<QT_Q2_K>(W, vocab, K, d_token, d_out, st, n);
    case QT_Q3_K:
    case QT_IQ3_S: return embed_go<QT_Q3_K>(W, vocab, K, d_token, d_out, st, n);
    case QT_Q4_K: return embed_go<QT_Q4_K>(W, vocab, K, d_token, d_out, st, n);
    case QT_Q5_K: return embed_go<QT_Q5_K>(W, vocab, K, d_token, d_out, st, n);
    case QT_Q6_K: return embed_go<QT_Q6_K>(W, vocab, K, d_token, d_out, st, n);
    default: return 0;
    }
}

template <int QT, int SEM>
static int dq_go(const void *W, int M, int K, float *out, cudaStream_t st)
{
    constexpr Geom g = geom_of(QT);
    const unsigned long long row_bytes = static_cast<unsigned long long>(K / g.block_weights) * g.block_bytes;
    const unsigned long long nchunk = (static_cast<unsigned long long>(M) * K + 7) / 8;
    unsigned long long blocks = (nchunk + 255) / 256;
    if (blocks > 148ull * 16) blocks = 148ull * 16;
    k_dequant<QT, SEM><<<static_cast<unsigned>(blocks), 256, 0, st>>>(
        static_cast<const uint8_t *>(W), M, K, row_bytes, out);
    return cudaGetLastError() == cudaSuccess ? 1 : 0;
}

int dq_launch(const void *W, int qtype, int M, int K, float *d_out, int sem, cudaStream_t st)
{
    const NvtxRange nvtx("tb.dequant");
    const Geom g = geom_of(qtype);
    if (!g.block_weights || !W || !d_out || M <= 0 || K <= 0 || K % g.block_weights) return 0;
    if (reinterpret_cast<uintptr_t>(d_out) & 15u) return 0;
    if (sem != 0 && sem != 1) return 0;
    switch (qtype) {
    case QT_F32: return dq_go<QT_F32, 0>(W, M, K, d_out, st);
    case QT_F16: return dq_go<QT_F16, 0>(W, M, K, d_out, st);
    case QT_BF16: return dq_go<QT_BF16, 0>(W, M, K, d_out, st);
    case QT_Q4_0: return dq_go<QT_Q4_0, 0>(W, M, K, d_out, st);
    case QT_Q8_0: return dq_go<QT_Q8_0, 0>(W, M, K, d_out, st);
    case QT_Q8_K: return dq_go<QT_Q8_K, 0>(W, M, K, d_out, st);
    case QT_Q2_K: return dq_go<QT_Q2_K, 0>(W, M, K, d_out, st);
    case QT_Q3_K:
    case QT_IQ3_S: return dq_go<QT_Q3_K, 0>(W, M, K, d_out, st);
    case QT_Q6_K: return dq_go<QT_Q6_K, 0>(W, M, K, d_out, st);
    case QT_Q4_K: return sem ? dq_go<QT_Q4_K, 1>(W, M, K, d_out, st) : dq_go<QT_Q4_K, 0>(W, M, K, d_out, st);
    case QT_Q5_K: return sem ? dq_go<QT_Q5_K, 1>(W, M, K, d_out, st) : dq_go<QT_Q5_K, 0>(W, M, K, d_out, st);
    default: return 0;
    }
}

}  // namespace tb
