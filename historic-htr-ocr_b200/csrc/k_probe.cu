// k_probe.cu — a test hook for the bounded device waits: every kernel of the library waits on mbarriers through
// mbar_wait (common.cuh), which gives up after a limit, flags DEV_TIMEOUT and returns false instead of spinning
// forever. This kernel makes such a wait run out on purpose — an mbarrier whose expected transaction never arrives —
// so a test can check, without hanging or faulting the GPU, that the flag reaches the host as OCR_ERR_DEVICE and that
// the context stays usable.
#include "kernels.cuh"

namespace ocr {

__global__ void k_wait_probe(int* err, uint32_t tries, int* waited_out) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
        mbar_expect_tx(&bar, 16);  // the one arrival comes, its 16 bytes never do: the phase stays open
    }
    __syncthreads();
    if (threadIdx.x == 0) *waited_out = mbar_wait(&bar, 0, err, tries, 1000) ? 0 : 1;
}

void launch_wait_probe(cudaStream_t st, int* err, uint32_t tries, int* waited_out) {
    k_wait_probe<<<1, 32, 0, st>>>(err, tries, waited_out);
}

}  // namespace ocr
