// Host-side CTC helpers with the reference signatures
// (include/turbo_ocr/recognition/ctc_decode.h:10-23 in TurboOCR).
#include "turbo_ocr/recognition/ctc_decode.h"

#include <fstream>

#define TOCR_SHIM_API __attribute__((visibility("default")))

namespace turbo_ocr::recognition {

TOCR_SHIM_API std::pair<std::string, float> ctc_greedy_decode(
    const int *indices, const float *scores, int seq_len,
    const std::vector<std::string> &label_list) {
  std::string text;
  float total = 0.0f;
  int emitted = 0;
  int prev = -1;
  const int n_labels = static_cast<int>(label_list.size());
  for (int t = 0; t < seq_len; ++t) {
    const int idx = indices[t];
    if (idx != prev && idx != 0 && idx < n_labels) {
      text.append(label_list[idx]);
      total += scores[t];
      ++emitted;
    }
    prev = idx;
  }
  return {text, emitted > 0 ? total / emitted : 0.0f};
}

TOCR_SHIM_API std::pair<std::string, float> ctc_greedy_decode_raw(
    const float *logits, int seq_len, int num_classes,
    const std::vector<std::string> &label_list) {
  std::string text;
  float total = 0.0f;
  int emitted = 0;
  int prev = -1;
  const int n_labels = static_cast<int>(label_list.size());
  for (int t = 0; t < seq_len; ++t) {
    const float *row = logits + static_cast<size_t>(t) * num_classes;
    int idx = 0;
    float best = row[0];
    for (int j = 1; j < num_classes; ++j)
      if (row[j] > best) {
        best = row[j];
        idx = j;
      }
    if (idx != prev && idx != 0 && idx < n_labels) {
      text.append(label_list[idx]);
      total += best;
      ++emitted;
    }
    prev = idx;
  }
  return {text, emitted > 0 ? total / emitted : 0.0f};
}

TOCR_SHIM_API std::string ctc_tokens_to_text(const int *tokens, int n_tokens,
                                             const std::vector<std::string> &label_list) {
  std::string text;
  const int n_labels = static_cast<int>(label_list.size());
  for (int k = 0; k < n_tokens; ++k)
    if (tokens[k] > 0 && tokens[k] < n_labels) text.append(label_list[tokens[k]]);
  return text;
}

TOCR_SHIM_API bool load_label_dict(const std::string &dict_path,
                                   std::vector<std::string> &label_list) {
  std::ifstream in(dict_path);
  if (!in) return false;
  std::string line;
  while (std::getline(in, line)) {
    // At most one '\n', then at most one '\r' (a "\r\r" line keeps one '\r'),
    // as the reference loader does (src/recognition/ctc_decode.cpp:150-154).
    if (!line.empty() && line.back() == '\n') line.pop_back();
    if (!line.empty() && line.back() == '\r') line.pop_back();
    label_list.push_back(std::move(line));
  }
  label_list.emplace_back(" ");
  return true;
}

}  // namespace turbo_ocr::recognition
