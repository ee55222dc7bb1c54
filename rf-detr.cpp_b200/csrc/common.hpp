// Logging and status helpers shared by the host code of librfdetr.
#pragma once

#include "rfdetr.h"

#include <cuda_runtime.h>

#include <exception>
#include <new>

// printf-style log through the process-global callback installed with
// rfdetr_set_log_callback (reference semantics: src/common.cpp:33-60).
void rfdetr_logf(rfdetr_log_level lvl, const char* fmt, ...)
#if defined(__GNUC__)
    __attribute__((format(printf, 2, 3)))
#endif
    ;

// Logs a CUDA error with context; returns true if `e` is an error.
bool rfdetr_cuda_failed(cudaError_t e, const char* what, const char* file, int line);

#define RFB_CUDA_FAIL(expr) rfdetr_cuda_failed((expr), #expr, __FILE__, __LINE__)

// Runs the body of a C entry point.  C++ exceptions must not cross the C ABI:
// an allocation failure returns `on_oom`, any other exception `on_error`, both
// logged through the callback.
template <class F, class R>
R rfdetr_c_boundary(F&& body, R on_oom, R on_error) noexcept {
    try {
        return body();
    } catch (const std::bad_alloc&) {
        rfdetr_logf(RFDETR_LOG_ERROR, "out of memory");
        return on_oom;
    } catch (const std::exception& e) {
        rfdetr_logf(RFDETR_LOG_ERROR, "unexpected error: %s", e.what());
        return on_error;
    } catch (...) {
        rfdetr_logf(RFDETR_LOG_ERROR, "unexpected error");
        return on_error;
    }
}

// The same for entry points that return a pointer and report through a status
// out-parameter: nullptr, with *st = RFDETR_ERR_OUT_OF_MEMORY or `on_error`.
template <class T, class F>
T* rfdetr_c_boundary_ptr(F&& body, rfdetr_status* st, rfdetr_status on_error) noexcept {
    try {
        return body();
    } catch (const std::bad_alloc&) {
        rfdetr_logf(RFDETR_LOG_ERROR, "out of memory");
        if (st) *st = RFDETR_ERR_OUT_OF_MEMORY;
    } catch (const std::exception& e) {
        rfdetr_logf(RFDETR_LOG_ERROR, "unexpected error: %s", e.what());
        if (st) *st = on_error;
    } catch (...) {
        rfdetr_logf(RFDETR_LOG_ERROR, "unexpected error");
        if (st) *st = on_error;
    }
    return nullptr;
}
