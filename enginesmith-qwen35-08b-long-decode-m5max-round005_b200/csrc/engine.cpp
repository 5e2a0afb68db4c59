// `engine --model MODEL_DIR`: the EngineSmith token-ID protocol over
// stdin/stdout JSON lines (docs/protocol.md; host loop of source/src/main.rs).
//
//   {"id":1,"op":"hello"}                          -> {"id":1,"ok":true,"protocol":1}
//   {"id":2,"op":"generate","prompt":[..],"max_tokens":n,"reset":true|false}
//                                                  -> {"id":2,"ok":true,"tokens":[..]}
//   failure                                        -> {"id":..,"ok":false,"error":"text"}
//
// A reader thread feeds request lines through a one-slot queue and, at end of
// input, cancels the running request (main.rs:17-25); replies go to stdout
// only, diagnostics to stderr.
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <iostream>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "q35.h"
#include "q35_json.h"

namespace {

struct LineQueue {
  std::mutex mu;
  std::condition_variable cv;
  std::deque<std::string> q;
  bool closed = false;
  void push(std::string s) {
    std::unique_lock<std::mutex> lk(mu);
    cv.wait(lk, [&] { return q.size() < 1 || closed; });
    q.push_back(std::move(s));
    cv.notify_all();
  }
  bool pop(std::string& s) {
    std::unique_lock<std::mutex> lk(mu);
    cv.wait(lk, [&] { return !q.empty() || closed; });
    if (q.empty()) return false;
    s = std::move(q.front());
    q.pop_front();
    cv.notify_all();
    return true;
  }
  void close() {
    std::lock_guard<std::mutex> lk(mu);
    closed = true;
    cv.notify_all();
  }
};

// Q35_ENGINE_TRACE=1: milliseconds from the end of input to each shutdown
// step, on stderr (diagnostics only).
std::atomic<int64_t> g_eof_ns{0};
bool trace_on() {
  static const bool on = std::getenv("Q35_ENGINE_TRACE") != nullptr;
  return on;
}
int64_t now_ns() {
  return std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}
void trace(const char* what) {
  if (trace_on() && g_eof_ns.load())
    std::fprintf(stderr, "engine: %s %.2f ms after end of input\n", what, (now_ns() - g_eof_ns.load()) * 1e-6);
}

std::string error_reply(const std::string& id, const std::string& msg) {
  std::string out = "{\"id\":" + id + ",\"ok\":false,\"error\":";
  q35json::escape(msg, out);
  out += "}";
  return out;
}

}  // namespace

int main(int argc, char** argv) {
  const char* model = nullptr;
  int device = 0;
  q35_opts opts = {};
  // Prompts take the tensor-core route by default, as the reference's prefill
  // takes its GEMM/flash-attention route (model.rs:100-110, :189-198).
  opts.flags = Q35_FLAG_TENSOR_PROMPT;
  for (int i = 1; i < argc; ++i) {
    std::string a = argv[i];
    if (a == "--model" && i + 1 < argc) model = argv[++i];
    else if (a == "--device" && i + 1 < argc) device = std::atoi(argv[++i]);
    else if (a == "--capacity" && i + 1 < argc) opts.capacity = uint32_t(std::strtoul(argv[++i], nullptr, 10));
    else if (a == "--tensor-prompt") opts.flags |= Q35_FLAG_TENSOR_PROMPT;  // the default, kept for old callers
    else if (a == "--decode-prompt") opts.flags &= ~Q35_FLAG_TENSOR_PROMPT;  // prompts through the decode kernels
    else {
      std::fprintf(stderr, "engine: unknown argument %s\n", a.c_str());
      return 1;
    }
  }
  if (!model) {
    std::fprintf(stderr, "engine: --model MODEL_DIR required\n");
    return 1;
  }
  q35_session* s = nullptr;
  char err[1024] = {0};
  if (q35_open(model, device, &opts, &s, err, sizeof err) != Q35_OK) {
    std::fprintf(stderr, "engine: %s\n", err);
    return 1;
  }
  // The queue and flag outlive main's loop: the detached reader may still be
  // closing the queue when main returns.
  static std::atomic<bool> eof{false};
  LineQueue& lines = *new LineQueue();
  std::thread reader([s, &lines] {
    std::string line;
    while (std::getline(std::cin, line)) lines.push(line);
    // Disconnect stops inference after the currently queued GPU work. The
    // cancel is published before the flag, so main never frees the session
    // while the reader still uses it.
    g_eof_ns.store(now_ns());
    q35_cancel(s);
    eof.store(true);
    lines.close();
  });
  reader.detach();

  std::string line;
  std::vector<uint32_t> prompt, tokens;
  while (lines.pop(line)) {
    if (eof.load()) break;  // main.rs:39
    q35json::Value req;
    std::string perr;
    std::string id = "null";
    std::string reply;
    if (!q35json::parse(line, req, perr) || req.type != q35json::Value::Object) {
      reply = error_reply(id, "invalid request: " + perr);
    } else {
      if (const q35json::Value* v = req.get("id")) {
        id.clear();
        q35json::dump(*v, id);
      }
      const q35json::Value* op = req.get("op");
      if (!op || op->type != q35json::Value::String) {
        reply = error_reply(id, "missing op");
      } else if (op->str == "hello") {
        reply = "{\"id\":" + id + ",\"ok\":true,\"protocol\":1}";
      } else if (op->str == "generate") {
        const q35json::Value* p = req.get("prompt");
        const q35json::Value* mt = req.get("max_tokens");
        const q35json::Value* rs = req.get("reset");
        uint64_t count = 0;
        std::string bad;
        prompt.clear();
        if (!p || p->type != q35json::Value::Array) bad = "missing prompt";
        else {
          prompt.reserve(p->arr.size());
          for (auto& x : p->arr) {
            uint64_t t;
            if (!x.as_u64(t) || t > 0xffffffffull) {
              bad = "invalid token";
              break;
            }
            prompt.push_back(uint32_t(t));
          }
        }
        if (bad.empty() && (!mt || !mt->as_u64(count))) bad = "missing max_tokens";
        if (bad.empty() && (!rs || rs->type != q35json::Value::Bool)) bad = "missing reset";
        // model.rs:98: the output length is checked before anything is
        // allocated for it
        if (bad.empty() && (count == 0 || count > uint64_t(q35_capacity(s)))) bad = "invalid output length";
        if (!bad.empty()) {
          reply = error_reply(id, bad);
        } else {
          tokens.assign(size_t(count), 0);
          int rc = q35_generate(s, prompt.data(), prompt.size(), size_t(count), rs->b ? 1 : 0,
                                tokens.data());
          if (eof.load()) {
            trace("request stopped");
            break;
          }
          if (rc != Q35_OK) {
            reply = error_reply(id, q35_last_error(s));
          } else {
            reply.reserve(32 + 8 * size_t(count));
            reply = "{\"id\":" + id + ",\"ok\":true,\"tokens\":[";
            for (uint64_t i = 0; i < count; ++i) {
              if (i) reply += ',';
              reply += std::to_string(tokens[size_t(i)]);
            }
            reply += "]}";
          }
        }
      } else {
        reply = error_reply(id, "unknown operation " + op->str);
      }
    }
    if (eof.load()) break;  // main.rs:45
    reply += '\n';
    std::fwrite(reply.data(), 1, reply.size(), stdout);
    std::fflush(stdout);
  }
  // End of input: the running request has drained (q35_generate waits for
  // its queued work, at most two graph launches). Freeing the session before
  // leaving makes the CUDA context's teardown at exit shorter (measured
  // ~0.2 s against ~0.3 s when the driver reclaims everything at exit).
  trace("loop left");
  q35_close(s);
  trace("session closed");
  return 0;
}
