// b200q_quantize_noalloc (include/b200q.h): the activation quantizer of the GEMV passes for callers that hold no
// b200q context and may not allocate device memory. The quantize kernel is the one the passes use (launch_quantize);
// its scratch — the quants, scales and block sums it writes before they are copied to the caller — is a fixed
// array in device memory that the library image carries, one per device, instead of a context's allocation.
//
// Every pointer the kernel reads is checked on the host before the launch: x and norm_w must be device (or managed)
// memory of `device`, 4-byte aligned (the kernel reads them as floats), and hold n floats inside their allocation;
// the stream must belong to `device`. A pointer that fails any check is rejected with B200Q_ERR_ARG, so it never
// reaches the GPU.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
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
// Per device: the scratch's device address, resolved with that device current, and the id of the CUDA context it
// was resolved in (a device reset makes a new primary context, whose id differs, and the address is resolved again).
struct ScratchAddr {
    void *ptr = nullptr;
    unsigned long long ctx_id = 0;
};
ScratchAddr g_addr[kMaxDevices];

// Driver entry points (through the runtime, no link-time dependency on libcuda): the allocation range of a pointer
// and the current context's id. Null when the driver does not provide them.
typedef CUresult (*PtrAttrFn)(void *, CUpointer_attribute, CUdeviceptr);
typedef CUresult (*CtxCurFn)(CUcontext *);
typedef CUresult (*CtxIdFn)(CUcontext, unsigned long long *);
PtrAttrFn g_ptr_attr = nullptr;
CtxCurFn g_ctx_cur = nullptr;
CtxIdFn g_ctx_id = nullptr;
bool g_entry_done = false;

void load_entry_points() {
    if (g_entry_done) return;
    g_entry_done = true;
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuPointerGetAttribute", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
        g_ptr_attr = reinterpret_cast<PtrAttrFn>(f);
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
        g_ctx_cur = reinterpret_cast<CtxCurFn>(f);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
        g_ctx_id = reinterpret_cast<CtxIdFn>(f);
    cudaGetLastError();
}

// Id of the context current on this thread (0 when unknown).
unsigned long long current_ctx_id() {
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!g_ctx_cur || !g_ctx_id || g_ctx_cur(&ctx) != CUDA_SUCCESS || !ctx || g_ctx_id(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

int fail(char *msg, unsigned len, int code, const char *fmt, ...) {
    if (msg && len) {
        va_list ap;
        va_start(ap, fmt);
        std::vsnprintf(msg, len, fmt, ap);
        va_end(ap);
    }
    return code;
}

// 0 when p .. p + bytes is device (or managed) memory of `device`, 4-byte aligned and inside one allocation; else
// the reason in msg and B200Q_ERR_ARG.
int check_device_floats(const void *p, size_t bytes, int device, const char *what, char *msg, unsigned len) {
    if (reinterpret_cast<uintptr_t>(p) % 4)
        return fail(msg, len, B200Q_ERR_ARG, "quantize_noalloc: %s is not 4-byte aligned", what);
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return fail(msg, len, B200Q_ERR_ARG, "quantize_noalloc: %s is not a CUDA pointer", what);
    }
    if (at.type != cudaMemoryTypeDevice && at.type != cudaMemoryTypeManaged)
        return fail(msg, len, B200Q_ERR_ARG, "quantize_noalloc: %s is not device memory (it must be device memory of "
                    "device %d)", what, device);
    if (at.type == cudaMemoryTypeDevice && at.device != device)
        return fail(msg, len, B200Q_ERR_ARG, "quantize_noalloc: %s is device memory of device %d, not of device %d",
                    what, at.device, device);
    // the allocation's range: a call whose range cannot be checked is refused rather than launched
    CUdeviceptr start = 0;
    size_t size = 0;
    const CUdeviceptr dp = reinterpret_cast<CUdeviceptr>(p);
    if (!g_ptr_attr || g_ptr_attr(&start, CU_POINTER_ATTRIBUTE_RANGE_START_ADDR, dp) != CUDA_SUCCESS ||
        g_ptr_attr(&size, CU_POINTER_ATTRIBUTE_RANGE_SIZE, dp) != CUDA_SUCCESS || size == 0)
        return fail(msg, len, B200Q_ERR_ARG, "quantize_noalloc: the allocation range of %s cannot be determined", what);
    if (dp < start || dp - start > size || bytes > size - (dp - start))
        return fail(msg, len, B200Q_ERR_ARG, "quantize_noalloc: %s + %zu bytes runs past the end of its allocation",
                    what, bytes);
    return B200Q_OK;
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
    load_entry_points();
    int rc = check_device_floats(x, size_t(n) * 4, device, "x", err_msg, err_len);
    if (rc == B200Q_OK && norm_w) rc = check_device_floats(norm_w, size_t(n) * 4, device, "norm_w", err_msg, err_len);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (rc == B200Q_OK && st) {
        int sd = -1;
        if (cudaStreamGetDevice(st, &sd) != cudaSuccess) {
            cudaGetLastError();
            rc = fail(err_msg, err_len, B200Q_ERR_ARG, "quantize_noalloc: stream is not a valid CUDA stream");
        } else if (sd != device) {
            rc = fail(err_msg, err_len, B200Q_ERR_ARG, "quantize_noalloc: stream belongs to device %d, not %d", sd,
                      device);
        }
    }
    auto cuda = [&](cudaError_t r, const char *what) {
        if (r != cudaSuccess && rc == B200Q_OK)
            rc = fail(err_msg, err_len, B200Q_ERR_CUDA, "quantize_noalloc: %s: %s", what, cudaGetErrorString(r));
        return r == cudaSuccess;
    };
    // the scratch's device address: resolved once per device (and again after a device reset), with the device
    // current; the host-side symbol g_scratch itself is not a device address
    if (rc == B200Q_OK) {
        ScratchAddr &sa = g_addr[device];
        const unsigned long long id = current_ctx_id();
        if (!sa.ptr || id == 0 || id != sa.ctx_id) {
            void *p = nullptr;
            if (cuda(cudaGetSymbolAddress(&p, g_scratch), "cudaGetSymbolAddress")) {
                sa.ptr = p;
                sa.ctx_id = id ? id : current_ctx_id();
            }
        }
    }
    if (rc == B200Q_OK) {
        uint8_t *s = static_cast<uint8_t *>(g_addr[device].ptr);
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
