// b200q_quantize_noalloc (include/b200q.h): the activation quantizer of the GEMV passes for callers that hold no
// b200q context and may not allocate device memory. The quantize kernel is the one the passes use (launch_quantize);
// its scratch — the quants, scales and block sums it writes before they are copied to the caller — is a fixed
// array in device memory that the library image carries, one per device, instead of a context's allocation.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/b200q.h"
#include "kernel_args.h"
#include "launch.h"
#include "layout.h"
#include "plan.h"

namespace b200q {
namespace {

constexpr unsigned kN = B200Q_NOALLOC_MAX_N;
// [q: kN int8][d: kN/32 floats][s: kN/32 floats][b: kN/16 int32][d16: kN/16 uint16]: the largest of each output
// over Q8_0 (d, b per 32-block), Q8_1 (d, s, b per 32-block; d16 = d, s pairs) and Q8_K (d per 256, b per 16).
constexpr size_t kQOff = 0, kDOff = kN, kSOff = kDOff + kN / 32 * 4, kBOff = kSOff + kN / 32 * 4,
                 kD16Off = kBOff + kN / 16 * 4, kScratchBytes = kD16Off + kN / 16 * 2;
static_assert(kScratchBytes <= 32768, "the scratch stays modest");

// Written by every call before it is read back; nothing in it needs to start at zero.
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_scratch_addr[kMaxDevices] = {};  // per device, resolved by the first call on that device

int fail(char *msg, unsigned len, int code, const char *fmt, ...) {
    if (msg && len) {
        va_list ap;
        va_start(ap, fmt);
        std::vsnprintf(msg, len, fmt, ap);
        va_end(ap);
    }
    return code;
}

}  // namespace
}  // namespace b200q

using namespace b200q;

extern "C" B200Q_API int b200q_quantize_noalloc(int device, const float *x, unsigned n, unsigned format,
                                                const float *norm_w, float norm_eps, unsigned norm_flags,
                                                void *stream, int8_t *q, void *scales, int32_t *bsums,
                                                char *err_msg, unsigned err_len) {
    if (err_msg && err_len) err_msg[0] = '\0';
    if (!format_supported(format))
        return fail(err_msg, err_len, B200Q_ERR_ARG, "quantize_noalloc: unknown weight format %u", format);
    const unsigned act = act_type(format), block = act == 2 ? 256u : 32u;
    if (!x || n == 0 || n % block)
        return fail(err_msg, err_len, B200Q_ERR_ARG, "quantize_noalloc: n = %u is not a positive multiple of %u", n,
                    block);
    if (n > kN)
        return fail(err_msg, err_len, B200Q_ERR_ARG,
                    "quantize_noalloc: n = %u exceeds B200Q_NOALLOC_MAX_N = %u (the fixed scratch holds no more)", n, kN);
    if (device < 0 || device >= kMaxDevices)
        return fail(err_msg, err_len, B200Q_ERR_ARG, "quantize_noalloc: device %d out of range", device);

    std::lock_guard<std::mutex> lock(g_mu);
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e == cudaSuccess && prev != device) e = cudaSetDevice(device);
    if (e != cudaSuccess)
        return fail(err_msg, err_len, B200Q_ERR_CUDA, "quantize_noalloc: device %d: %s", device, cudaGetErrorString(e));
    int rc = B200Q_OK;
    auto cuda = [&](cudaError_t r, const char *what) {
        if (r != cudaSuccess && rc == B200Q_OK)
            rc = fail(err_msg, err_len, B200Q_ERR_CUDA, "quantize_noalloc: %s: %s", what, cudaGetErrorString(r));
        return r == cudaSuccess;
    };
    if (!g_scratch_addr[device]) {
        void *p = nullptr;
        if (cuda(cudaGetSymbolAddress(&p, g_scratch), "cudaGetSymbolAddress")) g_scratch_addr[device] = p;
    }
    if (rc == B200Q_OK) {
        uint8_t *s = static_cast<uint8_t *>(g_scratch_addr[device]);
        QuantArgs a;
        a.x = x;
        a.n = n;
        a.act = act;
        if (norm_w) {
            a.norm_w = norm_w;
            a.norm_eps = norm_eps;
            a.norm_mode = 8u | (norm_flags & 3u);
        }
        a.q = reinterpret_cast<int8_t *>(s + kQOff);
        a.d = reinterpret_cast<float *>(s + kDOff);
        a.s = reinterpret_cast<float *>(s + kSOff);
        a.b = reinterpret_cast<int32_t *>(s + kBOff);
        a.d16 = reinterpret_cast<uint16_t *>(s + kD16Off);
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        if (cuda(launch_quantize(a, st), "quantize launch")) {
            if (q) cuda(cudaMemcpyAsync(q, a.q, n, cudaMemcpyDeviceToHost, st), "copy q");
            if (scales) {
                const void *src = act == 2 ? static_cast<const void *>(a.d) : static_cast<const void *>(a.d16);
                const size_t bytes = act == 0 ? n / 32 * 2 : act == 1 ? n / 32 * 4 : n / 256 * 4;
                cuda(cudaMemcpyAsync(scales, src, bytes, cudaMemcpyDeviceToHost, st), "copy scales");
            }
            if (bsums)
                cuda(cudaMemcpyAsync(bsums, a.b, (act == 2 ? n / 16 : n / 32) * 4, cudaMemcpyDeviceToHost, st),
                     "copy block sums");
            cuda(cudaStreamSynchronize(st), "stream synchronize");
        }
    }
    if (prev != device) cudaSetDevice(prev);
    return rc;
}
