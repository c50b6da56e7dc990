// Host side of the overlap between consecutive decode-attention calls on one stream: the device
// byte ranges a call reads and writes, and whether a call may start streaming its pages before
// the previous call launched on the same stream has completed.  Plain C++ (no CUDA types), so
// the CPU tests compile it on its own.
#pragma once

#include <cstddef>
#include <cstdint>
#include <mutex>
#include <unordered_map>

namespace tp {

// Device byte range [lo, hi).
struct Span {
  uintptr_t lo, hi;
};

constexpr int kMaxSpans = 12;

// The ranges one call reads, or writes.  More ranges than fit are treated as overlapping
// everything, so an overflow can only make a call wait.
struct Spans {
  Span s[kMaxSpans];
  int n = 0;
  bool all = false;
  void add(const void* p, size_t bytes) {
    if (!p || !bytes) return;
    if (n < kMaxSpans) s[n++] = Span{uintptr_t(p), uintptr_t(p) + bytes};
    else all = true;
  }
  bool meets(const Spans& o) const {
    if (all || o.all) return true;
    for (int i = 0; i < n; ++i)
      for (int j = 0; j < o.n; ++j)
        if (s[i].lo < o.s[j].hi && o.s[j].lo < s[i].hi) return true;
    return false;
  }
};

// The buffers of one attention call (sizes in bytes; NULL pointers are skipped).
struct CallBuffers {
  const void* q = nullptr;             // query, read
  size_t q_bytes = 0;
  const void* pages = nullptr;         // page pool, read (written by a decode step's flush)
  size_t pages_bytes = 0;
  const void* radii_scales = nullptr;  // per-page radius scales, like the pool
  size_t radii_scales_bytes = 0;
  const void* tail_k = nullptr;        // dense tail, read (written by a decode step)
  const void* tail_v = nullptr;
  size_t tail_bytes = 0;               // each of tail_k, tail_v
  const void* d_state = nullptr;       // state words, read (advanced by a decode step)
  size_t state_bytes = 0;
  const void* out = nullptr;           // fp16 output or partials, written
  size_t out_bytes = 0;
  bool step = false;                   // a decode step: appends k_new / v_new first
  const void* k_new = nullptr;         // the new token, read by a decode step
  const void* v_new = nullptr;
  size_t new_bytes = 0;                // each of k_new, v_new
  const void* exchange = nullptr;      // this rank's exchange buffer (sharded call), or NULL
  size_t exchange_bytes = 0;
};

// What `b` reads and writes.  The workspace is left out of both sides: the page pass writes its
// partials only after griddepcontrol.wait, and the split combine reads them after its own.  A
// sharded call's split combine reads and advances the epoch in this rank's exchange buffer
// before its wait, so the buffer counts as read and written and two calls on one exchange
// never overlap (calls on different exchanges, one per layer, may); the other ranks' buffers
// are written only after the wait.
inline void call_spans(const CallBuffers& b, Spans& reads, Spans& writes) {
  reads.add(b.q, b.q_bytes);
  reads.add(b.pages, b.pages_bytes);
  reads.add(b.radii_scales, b.radii_scales_bytes);
  reads.add(b.tail_k, b.tail_bytes);
  reads.add(b.tail_v, b.tail_bytes);
  reads.add(b.d_state, b.state_bytes);
  writes.add(b.out, b.out_bytes);
  if (b.step) {
    reads.add(b.k_new, b.new_bytes);
    reads.add(b.v_new, b.new_bytes);
    writes.add(b.d_state, b.state_bytes);
    writes.add(b.tail_k, b.tail_bytes);
    writes.add(b.tail_v, b.tail_bytes);
    writes.add(b.pages, b.pages_bytes);
    writes.add(b.radii_scales, b.radii_scales_bytes);
  }
  reads.add(b.exchange, b.exchange_bytes);
  writes.add(b.exchange, b.exchange_bytes);
}

// The last call's writes per stream.  Only this library's kernels let a dependent grid start
// before they complete (griddepcontrol.launch_dependents), and any other kernel launched between
// two calls starts after the first has completed, so the one call to compare with is the
// previous one of this library on the same stream; work on other streams is ordered by events,
// which wait for completion.
class StreamLog {
 public:
  // True when nothing the previous call on `stream` writes is read by this call; records this
  // call's writes as the stream's last either way.
  bool independent(const void* stream, const Spans& reads, const Spans& writes) {
    std::lock_guard<std::mutex> lock(mu_);
    const auto it = last_.find(stream);
    const bool ok = it == last_.end() || !it->second.meets(reads);
    last_[stream] = writes;
    return ok;
  }

 private:
  std::mutex mu_;
  std::unordered_map<const void*, Spans> last_;
};

}  // namespace tp
