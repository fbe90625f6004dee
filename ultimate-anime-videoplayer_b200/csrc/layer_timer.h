// Per-layer-kind device timing with CUDA events on the launching stream (kb2_set_profiling /
// kb2_read_profile): the role of the reference's GpuTiming event pairs
// (src/gpu/cuda/backend/gpu_timing.h:1-40).
#pragma once

#include <string>
#include <vector>

#include "host_util.h"

namespace kb2 {

class LayerTimer {
 public:
  struct Record {
    std::string name;
    uint64_t launches = 0;
    double ms = 0.0, flops = 0.0, bytes = 0.0;
  };

  bool enabled() const { return on_; }
  void enable(bool on) { on_ = on; }

  int kind(const char* name) {
    for (size_t i = 0; i < kinds_.size(); ++i)
      if (kinds_[i].name == name) return static_cast<int>(i);
    kinds_.push_back(Record{name});
    return static_cast<int>(kinds_.size()) - 1;
  }

  Status begin(cudaStream_t stream) {
    if (!on_) return Status::Ok();
    KB2_TRY(take(&open_));
    return cuda_status(cudaEventRecord(open_, stream), "cudaEventRecord");
  }

  Status end(int kind, double flops, double bytes, cudaStream_t stream) {
    if (!on_) return Status::Ok();
    cudaEvent_t stop = nullptr;
    KB2_TRY(take(&stop));
    KB2_CUDA(cudaEventRecord(stop, stream));
    pending_.push_back(Pending{kind, open_, stop, flops, bytes});
    open_ = nullptr;
    return Status::Ok();
  }

  // Records accumulated since the last read (synchronises on the recorded events).
  Status read(std::vector<Record>& out) {
    for (const Pending& p : pending_) {
      KB2_CUDA(cudaEventSynchronize(p.stop));
      float ms = 0.0f;
      KB2_CUDA(cudaEventElapsedTime(&ms, p.start, p.stop));
      Record& k = kinds_[p.kind];
      k.launches += 1;
      k.ms += ms;
      k.flops += p.flops;  // sums here; averaged per launch below
      k.bytes += p.bytes;
      pool_.push_back(p.start);
      pool_.push_back(p.stop);
    }
    pending_.clear();
    out = kinds_;
    for (Record& r : out) {
      if (r.launches > 0) {
        r.flops /= static_cast<double>(r.launches);
        r.bytes /= static_cast<double>(r.launches);
      }
    }
    for (Record& k : kinds_) {
      k.launches = 0;
      k.ms = 0.0;
      k.flops = 0.0;
      k.bytes = 0.0;
    }
    return Status::Ok();
  }

  ~LayerTimer() {
    for (const Pending& p : pending_) {
      cudaEventDestroy(p.start);
      cudaEventDestroy(p.stop);
    }
    for (cudaEvent_t e : pool_) cudaEventDestroy(e);
  }

 private:
  struct Pending {
    int kind;
    cudaEvent_t start, stop;
    double flops, bytes;
  };
  Status take(cudaEvent_t* e) {
    if (!pool_.empty()) {
      *e = pool_.back();
      pool_.pop_back();
      return Status::Ok();
    }
    return cuda_status(cudaEventCreate(e), "cudaEventCreate");
  }

  bool on_ = false;
  std::vector<Record> kinds_;
  std::vector<Pending> pending_;
  std::vector<cudaEvent_t> pool_;
  cudaEvent_t open_ = nullptr;
};

}  // namespace kb2
