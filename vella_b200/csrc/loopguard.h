// Repetition-loop guard and runaway retry of the decode loop (host logic).
//
// Reference: Worker/Sources/MLXAudioSTT/NemotronTranscribe/NemotronTranscribeText.swift:
// 98-127 (NemotronTranscribeLoop.tail / cut: a tail of one block of at most 64 tokens
// repeated at least 20 times, the shortest block wins, the repetition start walked back),
// NemotronTranscribeModel.swift:296-302 (endsInLoop: checked when the output holds at least
// 20 tokens and a multiple of 4) and :436-443 (retryingRunaway: a draft-and-verify run
// that loops or reaches the token limit is decoded again plain greedy).
#pragma once

#include <vector>

namespace vella {

constexpr int kLoopMinRepeats = 20;
constexpr int kLoopMaxPeriod = 64;

struct LoopTail {
  bool found = false;
  int start = 0;
  int period = 0;
};

inline LoopTail loop_tail(const std::vector<int>& t, int min_repeats = kLoopMinRepeats, int max_period = kLoopMaxPeriod) {
  LoopTail r;
  const int n = static_cast<int>(t.size());
  if (min_repeats < 2) return r;
  for (int period = 1; period <= max_period && period * min_repeats <= n; ++period) {
    bool periodic = true;
    for (int i = 0; i < period * (min_repeats - 1); ++i) {
      if (t[n - 1 - i] != t[n - 1 - i - period]) {
        periodic = false;
        break;
      }
    }
    if (!periodic) continue;
    int start = n - period * min_repeats;
    while (start > 0 && t[start - 1] == t[start - 1 + period]) --start;
    r.found = true;
    r.start = start;
    r.period = period;
    return r;
  }
  return r;
}

// Tokens up to and including the first copy of a looping tail; returns whether one existed.
inline bool loop_cut(std::vector<int>& t) {
  const LoopTail l = loop_tail(t);
  if (!l.found) return false;
  t.resize(l.start + l.period);
  return true;
}

inline bool ends_in_loop(std::vector<int>& out) {
  if (static_cast<int>(out.size()) < kLoopMinRepeats || out.size() % 4 != 0) return false;
  return loop_cut(out);
}

}  // namespace vella
