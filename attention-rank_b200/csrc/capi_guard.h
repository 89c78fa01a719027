// Exception -> error-code mapping of the extern "C" boundary, shared by every translation unit
// that defines entry points. It is the C-ABI form of the reference's pybind translation of
// attnrank::Error into AttnRankError (attnrank/src/bindings.cpp:134): no exception crosses the
// boundary, every failure leaves a message for ar_last_error().
#pragma once

#include <new>
#include <stdexcept>
#include <string>

#include "../../include/attnrank_b200.h"
#include "engine.h"

namespace arb {

void set_last_error(const std::string& message);  // capi.cu: the thread's ar_last_error() text

// Runs `body` (which returns an AR_* code). arb::Error maps to AR_ERR_DEVICE when a kernel reported
// the failure, AR_ERR_CUDA for a CUDA or cuBLASLt failure, else AR_ERR_INVALID; a failed host
// allocation and any other exception map to AR_ERR_INTERNAL.
template <typename F>
int guarded_call(F&& body) {
  try {
    set_last_error("");
    return body();
  } catch (const Error& error) {
    const std::string what = error.what();
    set_last_error(what);
    if (what.find("device reported") != std::string::npos) return AR_ERR_DEVICE;
    if (what.find("CUDA error") != std::string::npos || what.find("cuBLASLt") != std::string::npos) {
      return AR_ERR_CUDA;
    }
    return AR_ERR_INVALID;
  } catch (const std::bad_alloc&) {
    set_last_error("host allocation failed");
    return AR_ERR_INTERNAL;
  } catch (const std::exception& error) {
    set_last_error(error.what());
    return AR_ERR_INTERNAL;
  }
}

}  // namespace arb
