// Minimal host FIFO standing in for the Catapult `ac_channel<T>` template, so that the reference's
// host sources (hls/prefill_only/*.cpp, compiled by oracle/Makefile into oracle/_ref/) build
// without the Catapult install. Only read/write/available/size are needed by the host paths that
// the reference's glue and stream tops use (qwen_prefill_host_wrapper.cpp, *_stream_top.cpp).
//
// TEST INFRASTRUCTURE ONLY: this header is part of the oracle build; no product code includes it.
#pragma once

#include <cstddef>
#include <deque>

template <typename T>
class ac_channel {
 public:
  T read() {
    T value = queue_.front();
    queue_.pop_front();
    return value;
  }
  void write(const T& value) { queue_.push_back(value); }
  bool available(unsigned int count) const { return queue_.size() >= count; }
  unsigned int size() const { return static_cast<unsigned int>(queue_.size()); }
  bool empty() const { return queue_.empty(); }

 private:
  std::deque<T> queue_;
};
