// Instantiations and launcher of the tensor-core decode kernel.
#include "tq_decode_mma.cuh"

#include <atomic>

namespace tq {

constexpr int kMaxDevices = 64;

static int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = 0;
  }
  return dev < 0 || dev >= kMaxDevices ? 0 : dev;
}

// The dynamic shared-memory opt-in is state of the function on one device
// (context), so it is made once per device that launches the kernel.
template <int D, int BITS, int NT, int NW>
static void* prepare() {
  static std::atomic<unsigned long long> done{0};
  const unsigned long long bit = 1ull << current_device();
  if (!(done.load(std::memory_order_acquire) & bit)) {
    cudaFuncSetAttribute(decode_mma_kernel<D, BITS, NT, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)RingCfg<D, BITS, NT, NW>::SMEM_BYTES);
    done.fetch_or(bit, std::memory_order_acq_rel);
  }
  return (void*)decode_mma_kernel<D, BITS, NT, NW>;
}

// Resident CTAs per SM, queried once per device.
template <int D, int BITS, int NT, int NW>
static int occupancy() {
  static std::atomic<int> cached[kMaxDevices];
  const int dev = current_device();
  const int c = cached[dev].load(std::memory_order_relaxed);
  if (c) return c;
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, prepare<D, BITS, NT, NW>(), NW * 32,
                                                    RingCfg<D, BITS, NT, NW>::SMEM_BYTES) != cudaSuccess ||
      blocks < 1) {
    cudaGetLastError();
    return mma_min_blocks<D, NW>();
  }
  cached[dev].store(blocks, std::memory_order_relaxed);
  return blocks;
}

// The decode grid is a programmatic dependent of whatever kernel precedes it
// on the stream: its CTAs may be scheduled while that kernel finishes (the
// previous step's split merge calls griddepcontrol.launch_dependents on
// entry), and the kernel waits (griddepcontrol.wait) before it reads any
// global memory, so the launch latency between steps is hidden.
template <int D, int BITS, int NT, int NW>
static void launch_one(const DecodeParams& p, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.splits, (unsigned)p.units);
  cfg.blockDim = dim3(NW * 32);
  cfg.dynamicSmemBytes = RingCfg<D, BITS, NT, NW>::SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  prepare<D, BITS, NT, NW>();
  cudaLaunchKernelEx(&cfg, decode_mma_kernel<D, BITS, NT, NW>, p);
}

template <int D, int BITS>
static void launch_mma(const DecodeParams& p, cudaStream_t st) {
  // wide CTAs exist for d <= 128 only (the planner never picks them for d = 256)
  if constexpr (D <= 128) {
    if (p.nw == kMmaWarpsWide) {
      if (p.G <= 8) launch_one<D, BITS, 1, kMmaWarpsWide>(p, st);
      else launch_one<D, BITS, 2, kMmaWarpsWide>(p, st);
      return;
    }
  }
  if (p.G <= 8) launch_one<D, BITS, 1, kMmaWarps>(p, st);
  else launch_one<D, BITS, 2, kMmaWarps>(p, st);
}

template <int D, int BITS>
static int blocks_for(int G, int nw) {
  if constexpr (D <= 128) {
    if (nw == kMmaWarpsWide) return G <= 8 ? occupancy<D, BITS, 1, kMmaWarpsWide>() : occupancy<D, BITS, 2, kMmaWarpsWide>();
  }
  return G <= 8 ? occupancy<D, BITS, 1, kMmaWarps>() : occupancy<D, BITS, 2, kMmaWarps>();
}

#define TQ_DISPATCH(D_, bits_, CALL)                                   \
  do {                                                                 \
    if (D_ == 64) {                                                    \
      if (bits_ == 2) CALL(64, 2); else if (bits_ == 3) CALL(64, 3); else CALL(64, 4); \
    } else if (D_ == 128) {                                            \
      if (bits_ == 2) CALL(128, 2); else if (bits_ == 3) CALL(128, 3); else CALL(128, 4); \
    } else {                                                           \
      if (bits_ == 2) CALL(256, 2); else if (bits_ == 3) CALL(256, 3); else CALL(256, 4); \
    }                                                                  \
  } while (0)

void launch_mma_dispatch(int D, int bits, const DecodeParams& p, cudaStream_t st) {
#define CALL_LAUNCH(d, b) launch_mma<d, b>(p, st)
  TQ_DISPATCH(D, bits, CALL_LAUNCH);
#undef CALL_LAUNCH
}

int mma_blocks_per_sm(int D, int bits, int G, int nw) {
  int r = 1;
#define CALL_OCC(d, b) r = blocks_for<d, b>(G, nw)
  TQ_DISPATCH(D, bits, CALL_OCC);
#undef CALL_OCC
  return r;
}

}  // namespace tq

#ifdef TQ_TRACE
// Development builds only: copy the decode kernels' step timeline to the host.
extern "C" int tq_trace_read_decode(void* host, size_t bytes) {
  const size_t n = bytes < sizeof(tq::g_trace_dec) ? bytes : sizeof(tq::g_trace_dec);
  return cudaMemcpyFromSymbol(host, tq::g_trace_dec, n) == cudaSuccess ? 0 : -1;
}
extern "C" int tq_trace_clear_decode() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, tq::g_trace_dec) != cudaSuccess) return -1;
  return cudaMemset(p, 0, sizeof(tq::g_trace_dec)) == cudaSuccess ? 0 : -1;
}
#endif
