// Internal definitions shared by the C ABI translation units of libvcsrmc.so.
#pragma once
#include <cstdint>
#include <new>
#include <stdexcept>
#include <string>

#include "vcsrmc.h"
#include "vcsrmc/csr.hpp"
#include "vcsrmc/vcsr_formats.hpp"

#define VCSRMC_EXPORT extern "C" __attribute__((visibility("default")))

struct vcsrmc_csr {
    vcsrmc::CSR csr;
};

struct vcsrmc_format {
    vcsrmc::VCSRMC v;
};

namespace vcsrmc {

// half_scale (src/vcsr_mc.cu:14-22) from the largest |value|, shared by the host and device builders.
float half_scale_from_absmax(float amax);

// Thread-local last error, reported through vcsrmc_last_error().
void set_last_error(int status, const std::string& msg);
int fail(int status, const std::string& msg);

// An exception whose status code the C ABI returns as is.
struct StatusError : std::runtime_error {
    int status;
    StatusError(int s, const std::string& m) : std::runtime_error(m), status(s) {}
};

// Runs fn() and converts exceptions into a status + last-error message.
template <class Fn>
int guarded(Fn&& fn) {
    try {
        fn();
        return VCSRMC_OK;
    } catch (const StatusError& e) {
        return fail(e.status, e.what());
    } catch (const std::bad_alloc&) {
        return fail(VCSRMC_OOM, "host allocation failed");
    } catch (const IoError& e) {
        return fail(VCSRMC_IO_ERR, e.what());
    } catch (const FormatError& e) {
        return fail(VCSRMC_FORMAT_ERR, e.what());
    } catch (const std::exception& e) {
        return fail(VCSRMC_INVALID_ARG, e.what());
    } catch (...) {
        return fail(VCSRMC_INTERNAL, "unknown exception");
    }
}

}  // namespace vcsrmc
