// oracle/ref_cuda_launch.c.cu — test and benchmark infrastructure only.
//
// Compiles the reference's own CUDA kernels (layer4/tb_gguf_dequant.cu, included
// unmodified from the reference tree by oracle/Makefile) and adds one launcher
// that runs them on caller-owned device pointers on a caller-given stream, at
// the reference's default geometry (tb_gguf_dequant.cu:373-384 with no
// oscillator snapshot: 128 threads, one CTA per row).  The reference's own
// tb_cuda_matvec_device (.cu:422-472) wraps the same launch in a synchronous
// x upload, a y download and two stream syncs, which hide the kernel time;
// this entry point lets bench.py time the kernels themselves, back to back in
// a CUDA graph, beside this repository's kernels on the same B200.
#include "tb_gguf_dequant.cu"

extern "C" int tbr_cuda_launch(const void *W, int qtype, int M, int K, const float *d_x, float *d_out,
                               void *stream)
{
    const int blk = 128, grd = M;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const uint8_t *Wd = static_cast<const uint8_t *>(W);
    switch (qtype) {   // the dispatch of tb_gguf_dequant.cu:447-460
    case 1: k_f16_matvec<<<grd, blk, 0, st>>>(reinterpret_cast<const uint16_t *>(Wd), M, K, d_x, d_out); break;
    case 12: k_q4k_matvec<<<grd, blk, 0, st>>>(Wd, M, K, d_x, d_out); break;
    case 13: k_q5k_matvec<<<grd, blk, 0, st>>>(Wd, M, K, d_x, d_out); break;
    case 11:
    case 21: k_q3k_matvec<<<grd, blk, 0, st>>>(Wd, M, K, d_x, d_out); break;
    case 14: k_q6k_matvec<<<grd, blk, 0, st>>>(Wd, M, K, d_x, d_out); break;
    case 2: k_q4_0_matvec<<<grd, blk, 0, st>>>(Wd, M, K, d_x, d_out); break;
    case 8: k_q8_0_matvec<<<grd, blk, 0, st>>>(Wd, M, K, d_x, d_out); break;
    case 15: k_q8k_matvec<<<grd, blk, 0, st>>>(Wd, M, K, d_x, d_out); break;
    case 30: k_bf16_matvec<<<grd, blk, 0, st>>>(reinterpret_cast<const uint16_t *>(Wd), M, K, d_x, d_out); break;
    case 0: k_f32_matvec<<<grd, blk, 0, st>>>(reinterpret_cast<const float *>(Wd), M, K, d_x, d_out); break;
    default: return 0;
    }
    return cudaGetLastError() == cudaSuccess ? 1 : 0;
}
