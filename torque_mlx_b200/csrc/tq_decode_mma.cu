// Instantiations and launcher of the tensor-core decode kernel.
#include "tq_decode_mma.cuh"

namespace tq {

template <int D, int BITS>
static void launch_mma(const DecodeParams& p, cudaStream_t st) {
  dim3 grid(p.splits, (unsigned)p.units);
  if (p.G <= 8) {
    constexpr size_t smem = MmaCfg<D, BITS, 1>::SMEM_BYTES;
    cudaFuncSetAttribute(decode_mma_kernel<D, BITS, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    decode_mma_kernel<D, BITS, 1><<<grid, kMmaWarps * 32, smem, st>>>(p);
  } else {
    constexpr size_t smem = MmaCfg<D, BITS, 2>::SMEM_BYTES;
    cudaFuncSetAttribute(decode_mma_kernel<D, BITS, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    decode_mma_kernel<D, BITS, 2><<<grid, kMmaWarps * 32, smem, st>>>(p);
  }
}


void launch_mma_dispatch(int D, int bits, const DecodeParams& p, cudaStream_t st) {
  if (D == 64) {
    if (bits == 2) launch_mma<64, 2>(p, st);
    else if (bits == 3) launch_mma<64, 3>(p, st);
    else launch_mma<64, 4>(p, st);
  } else if (D == 128) {
    if (bits == 2) launch_mma<128, 2>(p, st);
    else if (bits == 3) launch_mma<128, 3>(p, st);
    else launch_mma<128, 4>(p, st);
  } else {
    if (bits == 2) launch_mma<256, 2>(p, st);
    else if (bits == 3) launch_mma<256, 3>(p, st);
    else launch_mma<256, 4>(p, st);
  }
}

}  // namespace tq
