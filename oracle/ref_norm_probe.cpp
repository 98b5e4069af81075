// ref_norm_probe.cpp -- TEST INFRASTRUCTURE ONLY (parity checker).
//
// Compiles the reference's own kernel/qwen35_decoder.cpp (included from where
// it lies in the reference checkout; nothing is copied) as its own translation
// unit of oracle/_ref/libbreeze_ref.so, next to ref_probe.cpp's
// quantized_matmul.cpp, exactly as the reference's build_kernel.py links the
// two files into one library.  It exports one probe of a value the decoder
// keeps internal:
//
//   refprobe_rmsnorm  -- the decoder's rmsnorm (kernel/qwen35_decoder.cpp:133-141),
//                        the normalisation in front of every projection, which
//                        the CUDA library fuses into its activation quantizer;
//   refprobe_silu_mul -- the MLP's g1 = siluf(g1) * g2 (kernel/qwen35_decoder.cpp:
//                        129, 408), the down projection's input, which the CUDA
//                        library also fuses into its quantizer.
#include "qwen35_decoder.cpp"

extern "C" void refprobe_rmsnorm(float* out, const float* x, const float* w, int s, int H, float eps) {
    rmsnorm(out, x, w, s, H, eps);
}

extern "C" void refprobe_silu_mul(float* out, const float* g, const float* u, long long n) {
    for (long long i = 0; i < n; ++i) out[i] = siluf(g[i]) * u[i];
}
