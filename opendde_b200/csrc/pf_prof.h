// pf_prof.h -- launch counting and optional per-kernel CUDA-event timing.
//
// Every kernel launch in the library goes through PF_LAUNCH_SCOPE(stream, "name"): it bumps
// a process-wide launch counter and, when profiling is switched on (pf_set_option
// PF_OPT_PROFILE), records a CUDA event pair around the launch on the launching stream.
// pf_profile_report() resolves the pairs (synchronising on the last event) into per-kernel
// launch counts, total milliseconds and total algorithmic work.
//
// PF_LAUNCH_SCOPE_WORK(stream, "name", work, unit) also states the launch's algorithmic work,
// computed from its arguments: unit 'f' = flops of the contraction it performs (2 per
// multiply-add, over the rows, queries and keys this launch processes), 'b' = the minimum HBM
// bytes it must read and write. A Fold-CP rank's launches therefore carry that rank's share.
#pragma once
#include <cuda_runtime.h>

namespace pf {
namespace prof {

void on_launch_begin(cudaStream_t st, const char* name, double work, char unit);
void on_launch_end(cudaStream_t st);

struct Scope {
  cudaStream_t st;
  Scope(cudaStream_t s, const char* name, double work = 0.0, char unit = 0) : st(s) {
    on_launch_begin(s, name, work, unit);
  }
  ~Scope() { on_launch_end(st); }
};

}  // namespace prof
}  // namespace pf

#define PF_LAUNCH_SCOPE(st, name) ::pf::prof::Scope _pf_prof_scope_((st), (name))
#define PF_LAUNCH_SCOPE_WORK(st, name, work, unit) \
  ::pf::prof::Scope _pf_prof_scope_((st), (name), (double)(work), (unit))
