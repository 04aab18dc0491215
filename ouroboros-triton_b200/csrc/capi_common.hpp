// Error plumbing shared by every extern "C" entry point: a thread-local
// message plus a guard that turns C++ exceptions into status codes, so no
// exception ever crosses the C ABI.
#pragma once

#include <exception>
#include <string>

#include "ouroboros_b200.h"

namespace ouro {

void set_error(const std::string& msg);
void clear_error();

class CapiError : public std::exception {
 public:
  CapiError(int code, std::string msg) : code_(code), msg_(std::move(msg)) {}
  int code() const { return code_; }
  const char* what() const noexcept override { return msg_.c_str(); }

 private:
  int code_;
  std::string msg_;
};

[[noreturn]] inline void fail(int code, const std::string& msg) { throw CapiError(code, msg); }

}  // namespace ouro

// Runs `body` (a statement block) and maps exceptions to OURO_E* codes.
#define OURO_CAPI_GUARD(...)                                   \
  try {                                                        \
    ::ouro::clear_error();                                     \
    __VA_ARGS__;                                               \
    return OURO_OK;                                            \
  } catch (const ::ouro::CapiError& e) {                       \
    ::ouro::set_error(e.what());                               \
    return e.code();                                           \
  } catch (const ::ouro::AllocError& e) {                      \
    ::ouro::set_error(e.what());                               \
    return OURO_EALLOC;                                        \
  } catch (const std::exception& e) {                          \
    ::ouro::set_error(e.what());                               \
    return OURO_EINVAL;                                        \
  } catch (...) {                                              \
    ::ouro::set_error("unknown native error");                 \
    return OURO_EINVAL;                                        \
  }
