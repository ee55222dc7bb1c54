// Status strings and the process-global log callback (behaviour of the
// reference's src/common.cpp:17-60: callback swapped under a mutex, invoked
// outside it, messages formatted into a 1 KiB buffer).
#include "common.hpp"

#include <cstdarg>
#include <cstdio>
#include <mutex>

namespace {
std::mutex g_mu;
rfdetr_log_cb g_cb = nullptr;
void* g_user = nullptr;
}  // namespace

extern "C" const char* rfdetr_status_str(rfdetr_status s) {
    switch (s) {
        case RFDETR_OK: return "ok";
        case RFDETR_ERR_INVALID_ARG: return "invalid argument";
        case RFDETR_ERR_FILE_NOT_FOUND: return "file not found";
        case RFDETR_ERR_IO: return "i/o error";
        case RFDETR_ERR_OUT_OF_MEMORY: return "out of memory";
        case RFDETR_ERR_DECODE: return "image decode error";
        case RFDETR_ERR_MODEL_FORMAT: return "model format error";
        case RFDETR_ERR_MODEL_LOAD: return "model load error";
        case RFDETR_ERR_INFERENCE: return "inference error";
        case RFDETR_ERR_NOT_IMPLEMENTED: return "not implemented";
    }
    return "unknown error";
}

extern "C" void rfdetr_set_log_callback(rfdetr_log_cb cb, void* user_data) {
    std::lock_guard<std::mutex> lk(g_mu);
    g_cb = cb;
    g_user = user_data;
}

void rfdetr_logf(rfdetr_log_level lvl, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    const int n = std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (n < 0) return;
    rfdetr_log_cb cb;
    void* ud;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        cb = g_cb;
        ud = g_user;
    }
    if (cb) cb(lvl, buf, ud);
}

bool rfdetr_cuda_failed(cudaError_t e, const char* what, const char* file, int line) {
    if (e == cudaSuccess) return false;
    rfdetr_logf(RFDETR_LOG_ERROR, "CUDA error %s (%s) at %s:%d: %s", cudaGetErrorName(e), cudaGetErrorString(e), file,
                line, what);
    return true;
}
