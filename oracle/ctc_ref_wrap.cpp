// Test-infrastructure wrapper (oracle only): exposes the REFERENCE's own
// ctc_greedy_decode / ctc_greedy_decode_raw (src/recognition/ctc_decode.cpp,
// compiled unchanged from the reference tree by oracle/Makefile) over a C ABI.
// Token indices are recovered exactly from the decoded text by giving every
// dictionary entry a unique fixed-width label "%05d".
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <thread>
#include <vector>

#include "turbo_ocr/recognition/ctc_decode.h"

using turbo_ocr::recognition::ctc_greedy_decode;
using turbo_ocr::recognition::ctc_greedy_decode_raw;

namespace {
std::vector<std::string> g_labels;

void ensure_labels(int n) {
  if ((int)g_labels.size() == n) return;
  g_labels.clear();
  g_labels.reserve(n);
  char buf[16];
  for (int i = 0; i < n; ++i) {
    std::snprintf(buf, sizeof(buf), "%05d", i);
    g_labels.emplace_back(buf);
  }
}

int parse(const std::string &text, int *tokens) {
  const int n = (int)text.size() / 5;
  for (int k = 0; k < n; ++k) tokens[k] = std::atoi(text.substr(5 * k, 5).c_str());
  return n;
}
}  // namespace

extern "C" {

// Latch the reference's SIMD_CTC switch (read once per process image).
int ctc_ref_init(int simd) {
  setenv("SIMD_CTC", simd ? "1" : "0", 1);
  ensure_labels(2);
  float row[2] = {0.f, 1.f};
  (void)ctc_greedy_decode_raw(row, 1, 2, g_labels);
  return 0;
}

// ctc_greedy_decode_raw over one line of fp32 "probs" [T, V].
int ctc_ref_decode_raw(const float *probs, int T, int V, int num_labels, int *tokens,
                       float *score) {
  ensure_labels(num_labels);
  auto [text, s] = ctc_greedy_decode_raw(probs, T, V, g_labels);
  *score = s;
  return parse(text, tokens);
}

// ctc_greedy_decode over per-step (index, score).
int ctc_ref_decode(const int *indices, const float *scores, int T, int num_labels,
                   int *tokens, float *score) {
  ensure_labels(num_labels);
  auto [text, s] = ctc_greedy_decode(indices, scores, T, g_labels);
  *score = s;
  return parse(text, tokens);
}

// CPU baseline: the reference decode_raw over B lines plus, beside it, the
// max-softmax probability 1/sum(exp(x - max)) of every step, spread over
// n_threads std::threads. probs holds the fp32-converted logits [B, T, V].
void ctc_ref_decode_batch(const float *logits, int B, int T, int V, int num_labels,
                          int n_threads, int *tokens, int *lens, float *scores) {
  ensure_labels(num_labels);
  auto work = [&](int b0, int b1) {
    std::vector<float> probmax(T);
    for (int b = b0; b < b1; ++b) {
      const float *line = logits + (size_t)b * T * V;
      auto [text, s] = ctc_greedy_decode_raw(line, T, V, g_labels);
      float acc = 0.f;
      for (int t = 0; t < T; ++t) {
        const float *row = line + (size_t)t * V;
        float m = row[0];
        for (int j = 1; j < V; ++j) m = row[j] > m ? row[j] : m;
        float sum = 0.f;
        for (int j = 0; j < V; ++j) sum += std::exp(row[j] - m);
        probmax[t] = 1.f / sum;
        acc += probmax[t];
      }
      lens[b] = parse(text, tokens + (size_t)b * T);
      scores[b] = s + 0.f * acc;
    }
  };
  if (n_threads < 1) n_threads = 1;
  std::vector<std::thread> th;
  const int per = (B + n_threads - 1) / n_threads;
  for (int i = 0; i < n_threads; ++i) {
    const int b0 = i * per, b1 = std::min(B, b0 + per);
    if (b0 < b1) th.emplace_back(work, b0, b1);
  }
  for (auto &t : th) t.join();
}

}  // extern "C"
