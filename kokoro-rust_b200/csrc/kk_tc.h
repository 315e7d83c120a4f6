// tcgen05 (5th-generation tensor core) implicit-GEMM convolution for the BF16 precision mode.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include "kk_common.cuh"

namespace kk {

// Load-time bf16 operand image of one convolution / linear layer.
struct TcWeights {
  void* w = nullptr;   // device bf16 weight image (layout owned by kk_tc.cu)
  size_t bytes = 0;
  int cin = 0, cout = 0, K = 0;
  int cin_pad = 0, cout_pad = 0;
};

// True when the device can run the tcgen05 kernels (compute capability 10.x).
bool tc_available();
// Build the bf16 image of a torch-layout [cout][cin][K] f32 weight on the current device.
cudaError_t tc_make_weights(const float* w_torch, int cin, int cout, int K, TcWeights* out);
// Whether this convolution shape / mode runs on the tcgen05 kernel.
bool tc_supported(const ConvArgs& a, const TcWeights& t);
// Launch the tcgen05 convolution (same semantics as launch_conv_simt). `err` receives 2 if a
// bounded pipeline wait expires.
// `trace` (optional) receives cycle accounting of CTA 0 per pipeline role (16 counters).
cudaError_t tc_conv(const ConvArgs& a, const TcWeights& t, int* err, cudaStream_t st,
                    unsigned long long* trace = nullptr);

}  // namespace kk
