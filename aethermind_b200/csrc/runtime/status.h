// Status / StatusOr with the reference's status codes
// (include/aethermind/base/status.h:39-58, values equal to am_status_code).
#pragma once
#include <string>
#include <utility>
#include <variant>

#include "aethermind_b200.h"

namespace aethermind {

enum class StatusCode : uint8_t {
    kOk = 0,
    kCancelled,
    kUnknown,
    kInvalidArgument,
    kDeadlineExceeded,
    kNotFound,
    kAlreadyExists,
    kPermissionDenied,
    kResourceExhausted,
    kFailedPrecondition,
    kAborted,
    kOutOfRange,
    kUnimplemented,
    kInternal,
    kUnavailable,
    kDataLoss,
    kOverflow,
    kUnauthenticated
};
static_assert(static_cast<int>(StatusCode::kOutOfRange) == AM_STATUS_OUT_OF_RANGE);
static_assert(static_cast<int>(StatusCode::kUnauthenticated) == AM_STATUS_UNAUTHENTICATED);

class Status {
public:
    Status() = default;
    Status(StatusCode c, std::string m) : code_(c), msg_(std::move(m)) {}
    static Status Ok() { return {}; }
    static Status InvalidArgument(std::string m) { return {StatusCode::kInvalidArgument, std::move(m)}; }
    static Status NotFound(std::string m) { return {StatusCode::kNotFound, std::move(m)}; }
    static Status OutOfRange(std::string m) { return {StatusCode::kOutOfRange, std::move(m)}; }
    static Status FailedPrecondition(std::string m) { return {StatusCode::kFailedPrecondition, std::move(m)}; }
    static Status AlreadyExists(std::string m) { return {StatusCode::kAlreadyExists, std::move(m)}; }
    static Status ResourceExhausted(std::string m) { return {StatusCode::kResourceExhausted, std::move(m)}; }
    static Status Internal(std::string m) { return {StatusCode::kInternal, std::move(m)}; }
    static Status Unimplemented(std::string m) { return {StatusCode::kUnimplemented, std::move(m)}; }
    static Status Overflow(std::string m) { return {StatusCode::kOverflow, std::move(m)}; }
    static Status DeadlineExceeded(std::string m) { return {StatusCode::kDeadlineExceeded, std::move(m)}; }
    static Status Unavailable(std::string m) { return {StatusCode::kUnavailable, std::move(m)}; }
    static Status FromAm(am_status_code c, const char* m) {
        return c == AM_STATUS_OK ? Status() : Status(static_cast<StatusCode>(c), m ? m : "");
    }
    bool ok() const { return code_ == StatusCode::kOk; }
    StatusCode code() const { return code_; }
    am_status_code am_code() const { return static_cast<am_status_code>(code_); }
    const std::string& message() const { return msg_; }
    std::string ToString() const;

private:
    StatusCode code_ = StatusCode::kOk;
    std::string msg_;
};

template <typename T>
class StatusOr {
public:
    StatusOr(T v) : v_(std::move(v)) {}              // NOLINT
    StatusOr(Status s) : v_(std::move(s)) {}         // NOLINT
    bool ok() const { return std::holds_alternative<T>(v_); }
    const T& value() const { return std::get<T>(v_); }
    T& value() { return std::get<T>(v_); }
    Status status() const { return ok() ? Status::Ok() : std::get<Status>(v_); }

private:
    std::variant<T, Status> v_;
};

}  // namespace aethermind

#define AM_RETURN_IF_ERROR(expr)                 \
    do {                                         \
        ::aethermind::Status _st = (expr);       \
        if (!_st.ok()) return _st;               \
    } while (0)
