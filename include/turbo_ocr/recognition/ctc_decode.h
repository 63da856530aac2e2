// CTC decode entry points of the reference
// (include/turbo_ocr/recognition/ctc_decode.h:10-23 in TurboOCR).
// The B200 path decodes on the GPU (tocr_ctc_greedy_f16); these host functions
// turn its token indices into text with the same collapse rule and dictionary
// layout, for callers that hold per-step indices/scores.
#pragma once

#include <string>
#include <utility>
#include <vector>

namespace turbo_ocr::recognition {

// Collapse per-step (index, score): emit index when it differs from the
// previous step, is not blank (0) and is inside the dictionary; the score is
// the mean of the emitted step scores (0 when nothing is emitted).
[[nodiscard]] std::pair<std::string, float> ctc_greedy_decode(
    const int *indices, const float *scores, int seq_len,
    const std::vector<std::string> &label_list);

// ctc_decode.h:15-17 — per step the argmax of raw scores (first maximum), then
// the same collapse; the line score is the mean emitted maximum.
[[nodiscard]] std::pair<std::string, float> ctc_greedy_decode_raw(
    const float *logits, int seq_len, int num_classes,
    const std::vector<std::string> &label_list);

// Text of an already-collapsed token list (the GPU decode's output).
[[nodiscard]] std::string ctc_tokens_to_text(const int *tokens, int n_tokens,
                                             const std::vector<std::string> &label_list);

// Dictionary loader: appends one label per line (CR/LF stripped) and a
// trailing " " label. label_list normally starts as {"blank"}.
[[nodiscard]] bool load_label_dict(const std::string &dict_path,
                                   std::vector<std::string> &label_list);

}  // namespace turbo_ocr::recognition
