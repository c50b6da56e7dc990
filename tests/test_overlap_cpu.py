"""When may a decode-attention call overlap the previous call on its stream (CPU).

The page pass of a call streams before its grid-dependency wait only when the previous call of
the library on the same stream writes nothing the call reads (tp_overlap.h: ``call_spans`` and
``StreamLog``).  A wrong "independent" would let a page pass read a cache, a query or an
exchange epoch that the previous call is still writing, so the decision is checked here case by
case: a small C++ driver is compiled with g++ against the header and run.
"""

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "turbopolar_b200", "csrc")

DRIVER = r"""
#include <cstdio>
#include <cstdlib>
#include "tp_overlap.h"
using namespace tp;

static unsigned char mem[1 << 20];
static const void* at(size_t off) { return mem + off; }

// One cache (pool, scales, tail, state) at `base`, a query and an output.
static CallBuffers call(size_t base, size_t q, size_t out, bool step) {
  CallBuffers b;
  b.q = at(q); b.q_bytes = 8192;
  b.pages = at(base); b.pages_bytes = 40000;
  b.radii_scales = at(base + 40000); b.radii_scales_bytes = 512;
  b.tail_k = at(base + 41000); b.tail_v = at(base + 50000); b.tail_bytes = 8192;
  b.d_state = at(base + 60000); b.state_bytes = 24;
  b.out = at(out); b.out_bytes = 8192;
  if (step) { b.step = true; b.k_new = at(q + 9000); b.v_new = at(q + 10000); b.new_bytes = 256; }
  return b;
}

static bool run(StreamLog& log, const void* stream, const CallBuffers& b, int device = 0, uint64_t capture = 0,
                uint64_t thread = 0) {
  Spans r, w;
  call_spans(b, r, w);
  return log.independent(StreamKey{device, uintptr_t(stream), thread, capture}, r, w);
}

// The decision and whether the call's cache (state words, pages, radius scales) is final.
static bool run_probe(StreamLog& log, const void* stream, const CallBuffers& b, bool* cache_final) {
  Spans r, w, c;
  call_spans(b, r, w);
  cache_spans(b, c);
  return log.independent(StreamKey{0, uintptr_t(stream), 0, 0}, r, w, &c, cache_final);
}

// The decision and whether the call's workspace at `ws` is used by no call of the chain.
static bool run_ws(StreamLog& log, const void* stream, CallBuffers b, size_t ws, bool* ws_clear) {
  b.workspace = at(ws);
  b.workspace_bytes = 4096;
  Spans r, w, c, x;
  call_spans(b, r, w);
  cache_spans(b, c);
  workspace_spans(b, x);
  bool fin = false;
  return log.independent(StreamKey{0, uintptr_t(stream), 0, 0}, r, w, &c, &fin, &x, ws_clear);
}

#define CHECK(cond) do { if (!(cond)) { std::printf("FAIL line %d: %s\n", __LINE__, #cond); std::exit(1); } } while (0)

int main() {
  const void* s1 = &mem[0];
  const void* s2 = &mem[1];
  {  // the first call on a stream waits; then layers of a decode step (other caches, queries,
     // outputs) stream early
    StreamLog log;
    CHECK(!run(log, s1, call(0, 300000, 400000, true)));
    CHECK(run(log, s1, call(100000, 310000, 410000, true)));
    CHECK(run(log, s1, call(200000, 320000, 420000, true)));
  }
  {  // two decode steps on one cache: the second reads the state, tail and pool the first writes
    StreamLog log;
    run(log, s1, call(0, 300000, 400000, true));
    CHECK(!run(log, s1, call(0, 310000, 410000, true)));
  }
  {  // a call is compared with every call since the last one that waited, not only the previous
     // one: steps on caches A, B, C, then A again (A's step may not have completed yet)
    StreamLog log;
    run(log, s1, call(0, 300000, 400000, true));
    CHECK(run(log, s1, call(100000, 310000, 410000, true)));
    CHECK(run(log, s1, call(200000, 320000, 420000, true)));
    CHECK(!run(log, s1, call(0, 330000, 430000, true)));
    CHECK(run(log, s1, call(100000, 340000, 440000, false)));  // the chain restarted at A's step
  }
  {  // a decode step, then plain attention on the same cache: it reads what the step wrote
    StreamLog log;
    run(log, s1, call(0, 300000, 400000, true));
    CHECK(!run(log, s1, call(0, 310000, 410000, false)));
  }
  {  // plain attention twice on one cache writes only the outputs: independent
    StreamLog log;
    run(log, s1, call(0, 300000, 400000, false));
    CHECK(run(log, s1, call(0, 310000, 410000, false)));
  }
  {  // the query is an earlier call's output, whole or in part
    StreamLog log;
    run(log, s1, call(0, 300000, 400000, false));
    CHECK(!run(log, s1, call(100000, 400000, 410000, false)));
    run(log, s1, call(0, 300000, 420000, false));
    CHECK(!run(log, s1, call(100000, 420000 + 8191, 430000, false)));
    run(log, s1, call(0, 300000, 440000, false));
    CHECK(run(log, s1, call(100000, 440000 + 8192, 460000, false)));  // adjacent, not overlapping
  }
  {  // the new token of a step is the previous call's output
    StreamLog log;
    run(log, s1, call(0, 300000, 409000, false));
    CHECK(!run(log, s1, call(100000, 400000, 430000, true)));  // k_new at 409000
  }
  {  // the previous call's output lands in this call's tail or state words
    StreamLog log;
    run(log, s1, call(0, 300000, 100000 + 41000, false));
    CHECK(!run(log, s1, call(100000, 310000, 450000, false)));
    run(log, s1, call(0, 300000, 100000 + 60000 - 100, false));
    CHECK(!run(log, s1, call(100000, 320000, 460000, false)));
  }
  {  // streams are logged separately
    StreamLog log;
    run(log, s2, call(500000, 350000, 450000, true));
    run(log, s1, call(0, 300000, 400000, true));
    CHECK(run(log, s2, call(0, 310000, 410000, true)));
    CHECK(!run(log, s1, call(0, 320000, 420000, true)));
  }
  {  // one handle (the legacy default stream, 0) on two devices names two streams: a step on
     // device 1 must not replace device 0's entry, or device 0's next step on the same cache
     // would be judged independent of its previous one
    StreamLog log;
    const void* s0 = nullptr;
    run(log, s0, call(0, 300000, 400000, true), 0);
    run(log, s0, call(500000, 310000, 410000, true), 1);
    CHECK(!run(log, s0, call(0, 320000, 420000, true), 0));
    CHECK(run(log, s0, call(600000, 330000, 430000, true), 1));
    CHECK(!run(log, s0, call(500000, 340000, 440000, true), 1));
  }
  {  // the per-thread default stream handle names one stream per host thread
    StreamLog log;
    run(log, s1, call(0, 300000, 400000, true), 0, 0, 11);
    run(log, s1, call(100000, 310000, 410000, true), 0, 0, 12);
    CHECK(!run(log, s1, call(0, 320000, 420000, true), 0, 0, 11));
    CHECK(run(log, s1, call(200000, 330000, 430000, true), 0, 0, 12));
  }
  {  // a capture starts its own chain (its first call waits), leaves the eager chain alone, and
     // replaces the stream's earlier captures
    StreamLog log;
    run(log, s1, call(0, 300000, 400000, true));
    CHECK(!run(log, s1, call(0, 310000, 410000, true), 0, 7));  // first call of capture 7
    CHECK(run(log, s1, call(100000, 320000, 420000, true), 0, 7));
    CHECK(!run(log, s1, call(0, 330000, 430000, true), 0, 7));  // same cache inside capture 7
    CHECK(!run(log, s1, call(0, 340000, 440000, true)));        // eager: the eager chain's step
    const size_t before = log.size();
    CHECK(!run(log, s1, call(100000, 350000, 450000, true), 0, 8));  // capture 8 replaces 7
    CHECK(log.size() == before);
  }
  {  // sharded calls: one exchange per layer overlaps, a shared exchange does not
    StreamLog log;
    CallBuffers a = call(0, 300000, 400000, true), b = call(100000, 310000, 410000, true);
    a.exchange = at(600000); a.exchange_bytes = 70000;
    b.exchange = at(700000); b.exchange_bytes = 70000;
    run(log, s1, a);
    CHECK(run(log, s1, b));
    CallBuffers c = call(200000, 320000, 420000, true);
    c.exchange = at(700000); c.exchange_bytes = 70000;
    CHECK(!run(log, s1, c));
  }
  {  // a chain longer than the log holds makes the next call wait and restarts the chain
    StreamLog log;
    run(log, s1, call(0, 300000, 400000, false));
    int waited = 0;
    for (int i = 0; i < 2 * ChainWrites::kMaxChain; ++i) {
      CallBuffers b = call(0, 300000, 400000 + 16 * (i % 4096), false);
      b.out_bytes = 16;
      if (!run(log, s1, b)) ++waited;
    }
    CHECK(waited >= 1 && waited <= 2);
  }
  {  // the cache probe of a dependent call: final when no call of the chain writes that cache
    StreamLog log;
    bool fin = true;
    CHECK(!run_probe(log, s1, call(0, 300000, 400000, true), &fin) && !fin);  // first call: unknown
    // Layer B's query is layer A's output (dependent), B's cache is written by nobody running.
    CHECK(!run_probe(log, s1, call(100000, 400000, 410000, true), &fin) && fin);
    // Layer C's query is B's output; B's step (in the chain) wrote B's cache, not C's.
    CHECK(!run_probe(log, s1, call(200000, 410000, 420000, false), &fin) && fin);
    // Attention on B's cache again: B's step is no longer in the chain (it restarted at C),
    // and C writes only its output.
    CHECK(run_probe(log, s1, call(100000, 300000, 430000, false), &fin) && fin);
    // A step on C's cache, then attention on it whose query is that step's output: dependent,
    // and the step (still running, perhaps) writes the cache.
    run_probe(log, s1, call(200000, 300000, 440000, true), &fin);
    CHECK(!run_probe(log, s1, call(200000, 440000, 450000, false), &fin) && !fin);
  }
  {  // workspaces: a call may write its partials before its wait only when it is independent
     // and no call of the chain (back to the last one that waited) uses an overlapping workspace
    StreamLog log;
    bool clear = true;
    CHECK(!run_ws(log, s1, call(0, 300000, 400000, true), 800000, &clear) && !clear);   // first call
    CHECK(run_ws(log, s1, call(100000, 310000, 410000, true), 810000, &clear) && clear);  // own workspace
    CHECK(run_ws(log, s1, call(200000, 320000, 420000, true), 820000, &clear) && clear);
    // Another layer sharing the first layer's workspace: independent, but that workspace's
    // partials may still be read by the first call's split combine.
    CHECK(run_ws(log, s1, call(300000, 330000, 430000, true), 800000 + 4095, &clear) && !clear);
    // Adjacent to the second layer's workspace, not overlapping it.
    CHECK(run_ws(log, s1, call(500000, 640000, 440000, true), 810000 + 4096, &clear) && clear);
    // A dependent call (same cache as the second layer) waits first: never "clear", and the chain
    // of workspaces restarts with its own.
    CHECK(!run_ws(log, s1, call(100000, 350000, 450000, true), 830000, &clear) && !clear);
    CHECK(run_ws(log, s1, call(0, 360000, 460000, true), 800000, &clear) && clear);  // the old chain is done
    CHECK(run_ws(log, s1, call(200000, 370000, 470000, true), 830000, &clear) && !clear);
    // No workspace given: never clear.
    CHECK(run(log, s1, call(300000, 380000, 480000, false)));
  }
  {  // more ranges than fit count as overlapping everything
    Spans r, w;
    for (int i = 0; i < kMaxSpans + 1; ++i) r.add(at(1000 * i), 10);
    w.add(at(900000), 10);
    CHECK(r.all && r.meets(w) && w.meets(r));
    Spans e;
    CHECK(!e.meets(w));
  }
  std::printf("ok\n");
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_overlap_decisions(tmp_path):
    src = tmp_path / "overlap_driver.cpp"
    src.write_text(DRIVER)
    exe = tmp_path / "overlap_driver"
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", CSRC, str(src), "-o", str(exe)], check=True,
                   capture_output=True, timeout=120)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert res.returncode == 0 and res.stdout.strip() == "ok", res.stdout + res.stderr
