// prof.h -- optional per-stage CUDA-event timing inside libgta.
//
// When enabled (gta_profile_enable), each instrumented stage records a pair
// of CUDA events on the stream its kernels run on, together with the stage's
// algorithmic work (flops or bytes).  gta_profile_get() reads them back.
#pragma once

#include <string>
#include <vector>

#include <cuda_runtime.h>

namespace gta {

struct ProfRecord {
    std::string name;
    cudaEvent_t start = nullptr, stop = nullptr;
    double units = 0.0;  // algorithmic flops (distance GEMM) or bytes (the rest)
    unsigned long long* counters = nullptr;  // optional device counters of the stage (cudaMalloc'd)
    int n_counters = 0;
};

bool prof_enabled();
void prof_push(ProfRecord&& r);
void count_launches(long long n);  // this library's kernel launches (gta_launch_count)

class ProfScope {
public:
    ProfScope(const char* name, double units, cudaStream_t st) : st_(st)
    {
        if (!prof_enabled()) return;
        rec_.name = name;
        rec_.units = units;
        if (cudaEventCreate(&rec_.start) != cudaSuccess) return;
        if (cudaEventCreate(&rec_.stop) != cudaSuccess) return;
        cudaEventRecord(rec_.start, st_);
        on_ = true;
    }
    ~ProfScope()
    {
        if (!on_) return;
        cudaEventRecord(rec_.stop, st_);
        prof_push(std::move(rec_));
    }
    ProfScope(const ProfScope&) = delete;
    ProfScope& operator=(const ProfScope&) = delete;

    // Zeroed device counters reported with this record (null when profiling is off).
    unsigned long long* counters(int n)
    {
        if (!on_ || n <= 0) return nullptr;
        if (cudaMalloc(&rec_.counters, sizeof(unsigned long long) * n) != cudaSuccess) return nullptr;
        cudaMemsetAsync(rec_.counters, 0, sizeof(unsigned long long) * n, st_);
        rec_.n_counters = n;
        return rec_.counters;
    }

private:
    cudaStream_t st_;
    ProfRecord rec_;
    bool on_ = false;
};

}  // namespace gta
