// Exception types of the reference's host API (include/turbo_ocr/common/errors.h
// in TurboOCR). The C++ shims over the C-ABI map TOCR_ERR_* statuses to these,
// so callers' catch clauses keep working unchanged.
#pragma once
#include <stdexcept>
#include <string>

namespace turbo_ocr {

class OcrError : public std::runtime_error {
  using std::runtime_error::runtime_error;
};
class ModelLoadError : public OcrError {
  using OcrError::OcrError;
};
class InferenceError : public OcrError {
  using OcrError::OcrError;
};
class CudaError : public OcrError {
  using OcrError::OcrError;
};
class TimeoutError : public OcrError {
 public:
  TimeoutError() : OcrError("Inference timed out") {}
  explicit TimeoutError(const std::string &msg) : OcrError(msg) {}
};

// Throws the reference exception that corresponds to a C-ABI status.
void throw_on_status(int status, const char *where);

}  // namespace turbo_ocr
