// trace.h — what a context last queued on its GPU, and the debug-sync settings.
//
// The counterpart of the reference's GPUDebugSync (src/gpu/GPUDebugSync.hpp:5-22): every launch
// records its kernel name with one relaxed atomic store and a sequence number
// (note_gpu_kernel, src/gpu/GPUDebugSync.cpp:246-253), every C entry point records its phase (its
// own name) and opens an NVTX range of that name, and a failed or timed-out wait reports
// "<seq> <phase> <kernel>" of the last work queued. Off by default; the environment turns the
// rest on, read once:
//
//   ADAI_B200_SYNC=off|step|kernel|kernel:N   (the reference's ADAI_GPU_SYNC is read when unset)
//       step:     every entry point waits for its work before it returns
//       kernel:   also wait before every launch, so a failure is attributed to the one kernel
//                 that ran; the decode step then runs its kernels one by one instead of
//                 replaying its CUDA graph
//       kernel:N: wait before every Nth launch only
//   ADAI_B200_TRACE_FILE=<path>               (or ADAI_GPU_TRACE_FILE)
//       keep "<seq> <phase> <kernel>" of the last work in this file, rewritten in place, so a
//       process killed in a hang leaves it behind
//
// Values that cannot be read leave the setting at its default (off / no file).
#ifndef ADAI_B200_TRACE_H
#define ADAI_B200_TRACE_H

#include <atomic>
#include <string>

namespace adai_b200_trace {

enum SyncMode { kSyncOff = 0, kSyncStep = 1, kSyncKernel = 2 };

struct Settings {
    int mode = kSyncOff;
    unsigned every = 1;  // kSyncKernel: wait before every Nth launch
    std::string trace_file;
};

// Parses an ADAI_B200_SYNC value (null or empty = off). Returns false, with `problem` set and
// mode / every left at off / 1, for a value it cannot read.
bool parse_sync(const char* value, int* mode, unsigned* every, std::string* problem);

// The process's settings: from the environment on first use, or the last set_settings().
const Settings& settings();
// Replaces the process's settings (tests and tools); closes an open trace file.
void set_settings(const Settings& s);

struct WorkTrace {
    std::atomic<const char*> phase{"idle"};          // entry point running now
    std::atomic<const char*> kernel{"none"};         // last kernel queued
    std::atomic<const char*> kernel_phase{"idle"};   // entry point that queued it
    std::atomic<unsigned long long> seq{0};          // launches queued so far

    // Records one launch; writes the trace file when one is set.
    void note_kernel(const char* name);
    std::string describe() const;  // "<seq> <phase> <kernel>" of the last launch
};

// NVTX range of an entry point plus its phase tag (restored on exit, so an entry point called
// from another reports the inner one while it runs).
class PhaseScope {
   public:
    PhaseScope(WorkTrace* t, const char* name);
    ~PhaseScope();
    PhaseScope(const PhaseScope&) = delete;
    PhaseScope& operator=(const PhaseScope&) = delete;

   private:
    WorkTrace* t_;
    const char* prev_;
};

}  // namespace adai_b200_trace

#endif  // ADAI_B200_TRACE_H
