// trace.cu — host side of the work trace (declared in trace.h). Plain C++; the NVTX calls come
// from the header-only NVTX v3 in the CUDA toolkit and cost nothing unless a profiler attaches.
#include "trace.h"

#include <fcntl.h>
#include <unistd.h>

#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include <nvtx3/nvToolsExt.h>

namespace adai_b200_trace {
namespace {

std::mutex g_mu;       // settings and the trace file
Settings* g_settings;  // owned; replaced by set_settings
int g_fd = -1;         // open trace file

const char* env2(const char* a, const char* b) {
    const char* v = std::getenv(a);
    if (v && *v) return v;
    v = std::getenv(b);
    return (v && *v) ? v : nullptr;
}

void open_trace_locked(const std::string& path) {
    if (g_fd >= 0) ::close(g_fd);
    g_fd = -1;
    if (!path.empty()) g_fd = ::open(path.c_str(), O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
}

Settings* load_locked() {
    if (!g_settings) {
        auto* s = new Settings();
        std::string problem;
        if (!parse_sync(env2("ADAI_B200_SYNC", "ADAI_GPU_SYNC"), &s->mode, &s->every, &problem))
            std::fprintf(stderr, "adai_b200: %s (debug sync stays off)\n", problem.c_str());
        if (const char* f = env2("ADAI_B200_TRACE_FILE", "ADAI_GPU_TRACE_FILE")) s->trace_file = f;
        open_trace_locked(s->trace_file);
        g_settings = s;
    }
    return g_settings;
}

void write_trace(const std::string& line) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_fd < 0) return;
    const std::string text = line + "\n";
    // rewritten in place: whatever the process leaves behind is the last line written
    if (::pwrite(g_fd, text.data(), text.size(), 0) == static_cast<ssize_t>(text.size()) &&
        ::ftruncate(g_fd, static_cast<off_t>(text.size())) != 0) {
        // a trace that cannot be shortened keeps a stale tail; the first line is still current
    }
}

}  // namespace

bool parse_sync(const char* value, int* mode, unsigned* every, std::string* problem) {
    *mode = kSyncOff;
    *every = 1;
    if (!value || !*value) return true;
    const std::string v(value);
    if (v == "off" || v == "0") return true;
    if (v == "step") {
        *mode = kSyncStep;
        return true;
    }
    if (v == "kernel") {
        *mode = kSyncKernel;
        return true;
    }
    if (v.rfind("kernel:", 0) == 0) {
        const std::string n = v.substr(7);
        char* end = nullptr;
        errno = 0;
        const unsigned long k = n.empty() ? 0 : std::strtoul(n.c_str(), &end, 10);
        if (!n.empty() && n[0] != '-' && end && *end == '\0' && errno == 0 && k >= 1 &&
            k <= 1000000) {
            *mode = kSyncKernel;
            *every = static_cast<unsigned>(k);
            return true;
        }
        if (problem) *problem = "ADAI_B200_SYNC: '" + v + "' needs a count from 1 to 1000000";
        return false;
    }
    if (problem) *problem = "ADAI_B200_SYNC: '" + v + "' is not off, step, kernel or kernel:N";
    return false;
}

const Settings& settings() {
    std::lock_guard<std::mutex> lk(g_mu);
    return *load_locked();
}

void set_settings(const Settings& s) {
    std::lock_guard<std::mutex> lk(g_mu);
    // the previous object stays allocated: a reader may still hold a reference to it
    g_settings = new Settings(s);
    open_trace_locked(s.trace_file);
}

void WorkTrace::note_kernel(const char* name) {
    kernel.store(name, std::memory_order_relaxed);
    kernel_phase.store(phase.load(std::memory_order_relaxed), std::memory_order_relaxed);
    seq.fetch_add(1, std::memory_order_relaxed);
    if (!settings().trace_file.empty()) write_trace(describe());
}

std::string WorkTrace::describe() const {
    return std::to_string(seq.load(std::memory_order_relaxed)) + " " +
           kernel_phase.load(std::memory_order_relaxed) + " " +
           kernel.load(std::memory_order_relaxed);
}

PhaseScope::PhaseScope(WorkTrace* t, const char* name) : t_(t), prev_(nullptr) {
    nvtxRangePushA(name);
    if (t_) {
        prev_ = t_->phase.load(std::memory_order_relaxed);
        t_->phase.store(name, std::memory_order_relaxed);
    }
}

PhaseScope::~PhaseScope() {
    if (t_) t_->phase.store(prev_, std::memory_order_relaxed);
    nvtxRangePop();
}

}  // namespace adai_b200_trace
