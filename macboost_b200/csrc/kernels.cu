// Kernel dispatch and the row-major -> feature-major transpose.
#include "kernels_common.cuh"

namespace mb {
namespace {

// Row-major [rows][F] -> feature-major [F][ld], 32x32 tiles through shared
// memory (padded against bank conflicts).
__global__ void __launch_bounds__(256) transpose_kernel(const float* __restrict__ in,
                                                        long long rows, int F,
                                                        float* __restrict__ out, long long ld) {
  __shared__ float t[32][33];
  const long long r0 = static_cast<long long>(blockIdx.x) * 32;
  const int f0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const long long r = r0 + i;
    const int f = f0 + threadIdx.x;
    if (r < rows && f < F) t[i][threadIdx.x] = in[r * F + f];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int f = f0 + i;
    const long long r = r0 + threadIdx.x;
    if (r < rows && f < F) out[f * ld + r] = t[threadIdx.x][i];
  }
}

}  // namespace

cudaError_t launch_forest(int layout, bool planes, bool cat, const KArgs& a, size_t smem,
                          int grid, cudaStream_t stream, int code_bytes, const TopRecords* top) {
  if (layout == 2) return launch_codes(code_bytes, cat, a, smem, grid, stream, nullptr);
  const bool pay = layout == 3;
  if ((layout == 0 || pay) && top)
    return launch_complete_top(planes, cat, pay, a, *top, smem, grid, stream, nullptr);
  return (layout == 0 || pay) ? launch_complete(planes, cat, pay, a, smem, grid, stream, nullptr)
                              : launch_explicit(planes, cat, a, smem, grid, stream, nullptr);
}

cudaError_t forest_occupancy(int layout, bool planes, bool cat, int K, int G, int R,
                             size_t smem, int* ctas, int code_bytes, bool top) {
  KArgs a{};
  a.K = K;
  a.G = G;
  a.R = R;
  if (layout == 2) return launch_codes(code_bytes, cat, a, smem, 1, nullptr, ctas);
  const bool pay = layout == 3;
  if ((layout == 0 || pay) && top) {
    static TopRecords none{};
    return launch_complete_top(planes, cat, pay, a, none, smem, 1, nullptr, ctas);
  }
  return (layout == 0 || pay) ? launch_complete(planes, cat, pay, a, smem, 1, nullptr, ctas)
                              : launch_explicit(planes, cat, a, smem, 1, nullptr, ctas);
}

cudaError_t launch_transpose(const float* in, long long rows, int F, float* out, long long ld,
                             cudaStream_t stream) {
  if (rows <= 0 || F <= 0) return cudaSuccess;
  dim3 grid(unsigned((rows + 31) / 32), unsigned((F + 31) / 32));
  transpose_kernel<<<grid, dim3(32, 8), 0, stream>>>(in, rows, F, out, ld);
  return cudaGetLastError();
}

}  // namespace mb
