// Minimal stand-in for spdlog, used only to compile the reference engine's
// sources as a CPU oracle. spdlog is absent from this image and the reference
// sources only include it (one warning call in the CPU allocator); all
// functions here are no-ops.
#pragma once
#include <functional>
#include <memory>
#include <mutex>
#include <string>
namespace spdlog {
template<typename... A> inline void warn(A&&...) {}
template<typename... A> inline void info(A&&...) {}
template<typename... A> inline void error(A&&...) {}
template<typename... A> inline void debug(A&&...) {}
}  // namespace spdlog
