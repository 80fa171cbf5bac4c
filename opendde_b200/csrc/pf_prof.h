// pf_prof.h -- launch counting and optional per-kernel CUDA-event timing.
//
// Every kernel launch in the library goes through PF_LAUNCH_SCOPE(stream, "name"): it bumps
// a process-wide launch counter and, when profiling is switched on (pf_set_option
// PF_OPT_PROFILE), records a CUDA event pair around the launch on the launching stream.
// pf_profile_report() resolves the pairs (synchronising on the last event) into per-kernel
// launch counts and total milliseconds.
#pragma once
#include <cuda_runtime.h>

namespace pf {
namespace prof {

void on_launch_begin(cudaStream_t st, const char* name);
void on_launch_end(cudaStream_t st);

struct Scope {
  cudaStream_t st;
  Scope(cudaStream_t s, const char* name) : st(s) { on_launch_begin(s, name); }
  ~Scope() { on_launch_end(st); }
};

}  // namespace prof
}  // namespace pf

#define PF_LAUNCH_SCOPE(st, name) ::pf::prof::Scope _pf_prof_scope_((st), (name))
