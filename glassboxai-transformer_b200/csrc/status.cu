// status.cu -- status codes, per-thread error detail and cached device info.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <mutex>

#include "gbx_common.cuh"
#include "rows.cuh"

namespace gbx {

static thread_local char t_last_error[512] = "";

int set_error(int code, const char* fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_last_error, sizeof t_last_error, fmt, ap);
    va_end(ap);
    return code;
}

void clear_error() { t_last_error[0] = 0; }

int check_launch(const char* what)
{
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(GBX_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    return GBX_OK;
}

static constexpr int kMaxDevices = 64;
static DeviceInfo g_info[kMaxDevices];
static std::once_flag g_once[kMaxDevices];

int device_info(DeviceInfo* out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(GBX_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return set_error(GBX_ERANGE, "device ordinal %d", dev);
    std::call_once(g_once[dev], [dev] {
        int v = 0;
        g_info[dev].sm_count = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
            g_info[dev].sm_count = v;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) == cudaSuccess)
            g_info[dev].max_smem_optin = v;
    });
    if (g_info[dev].sm_count <= 0) return set_error(GBX_ECUDA, "could not query device %d", dev);
    *out = g_info[dev];
    return GBX_OK;
}

bool small_row_grid(int64_t ctas_at_256)
{
    DeviceInfo di;
    return device_info(&di) == GBX_OK && ctas_at_256 < (int64_t)kSmallGridCTAsPerSM * di.sm_count;
}

static std::atomic<int> g_pdl{0};

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }

static std::atomic<uint64_t> g_first_wait_ns{kDeviceWaitNs};

uint64_t first_wait_limit_ns() { return g_first_wait_ns.load(std::memory_order_relaxed); }

}  // namespace gbx

extern "C" {

int gbx_set_pdl(int enable) { return gbx::g_pdl.exchange(enable ? 1 : 0); }

uint64_t gbx_set_first_wait_limit(uint64_t ns) { return gbx::g_first_wait_ns.exchange(ns); }

int gbx_version(void) { return 100; }

const char* gbx_status_string(int status)
{
    switch (status) {
    case GBX_OK: return "GBX_OK";
    case GBX_EINVAL: return "GBX_EINVAL";
    case GBX_EDTYPE: return "GBX_EDTYPE";
    case GBX_ERANGE: return "GBX_ERANGE";
    case GBX_ECUDA: return "GBX_ECUDA";
    case GBX_EIO: return "GBX_EIO";
    case GBX_ENOTFOUND: return "GBX_ENOTFOUND";
    case GBX_ENOMEM: return "GBX_ENOMEM";
    default: return "GBX_E?";
    }
}

const char* gbx_last_error(void) { return gbx::t_last_error; }

}  // extern "C"
