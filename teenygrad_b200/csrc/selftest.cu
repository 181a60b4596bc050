// Self-test of the kernels' failure path: a bounded wait that runs out.
//
// Every mbarrier wait in the library gives up after a time limit (or as soon
// as another CTA has flagged an error), records its bit in the context's
// device error word and lets the kernel return, so a lost arrival never hangs
// the GPU.  tb_selftest_bounded_wait exercises exactly that code (mbar_wait_ns)
// on an mbarrier that nothing ever arrives on: CTA 0 waits with the caller's
// short limit and gives up; CTA 1 waits with the kernels' normal limit and
// must return early because CTA 0 flagged the error word.  No fault, trap or
// hang is involved; the context stays usable.
#include "common.cuh"

namespace tb {

__global__ void selftest_wait_kernel(int* err, unsigned long long short_ns, unsigned long long* elapsed_ns) {
    __shared__ __align__(8) uint64_t bar;
    const uint32_t b = smem_u32(&bar);
    if (threadIdx.x == 0) {
        mbar_init(b, 1);   // count 1, and nothing arrives
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned long long t0 = globaltimer();
        const bool ok = blockIdx.x == 0 ? mbar_wait_ns(b, 0, err, DEV_ERR_TIMEOUT_MISC, short_ns)
                                        : mbar_wait(b, 0, err, DEV_ERR_TIMEOUT_MISC);
        elapsed_ns[blockIdx.x] = ok ? 0ull : globaltimer() - t0;
    }
}

}  // namespace tb

using namespace tb;

extern "C" int tb_selftest_bounded_wait(tb_ctx* ctx, int limit_us, unsigned long long* elapsed_ns) {
    if (!ctx || !elapsed_ns) return TB_ERR_ARG;
    TB_REQUIRE(ctx, limit_us > 0 && limit_us <= 1000000, TB_ERR_ARG, "selftest: limit_us in (0, 1e6]");
    return launch(ctx, "selftest_wait", selftest_wait_kernel, dim3(2), dim3(32), 0, ctx->d_err,
                  (unsigned long long)limit_us * 1000ull, elapsed_ns);
}
