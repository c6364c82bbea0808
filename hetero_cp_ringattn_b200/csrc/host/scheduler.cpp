// Queue / active-set core of the iterative batch scheduler (rust/src/distributed/scheduler.rs:
// FIFO admission, at most max_batch_size active requests, removal on completion). The
// coordinator keeps the request objects; this core decides the order and the admission.
#include "hcp_host.h"

#include <algorithm>
#include <chrono>

namespace hcp::host {

BatchSchedulerCore::BatchSchedulerCore(int64_t max_batch_size) : max_batch_(max_batch_size) {
  if (max_batch_size < 1) throw std::invalid_argument("max_batch_size must be >= 1");
}

void BatchSchedulerCore::Enqueue(uint64_t request_id) {
  {
    std::lock_guard<std::mutex> g(mu_);
    pending_.push_back(request_id);
  }
  cv_.notify_all();
}

std::optional<uint64_t> BatchSchedulerCore::PopPending() {
  std::lock_guard<std::mutex> g(mu_);
  if (pending_.empty() || int64_t(active_.size()) >= max_batch_) return std::nullopt;
  const uint64_t id = pending_.front();
  pending_.pop_front();
  return id;
}

void BatchSchedulerCore::RequeueFront(uint64_t request_id) {
  {
    std::lock_guard<std::mutex> g(mu_);
    pending_.push_front(request_id);
  }
  cv_.notify_all();
}

void BatchSchedulerCore::Activate(uint64_t request_id) {
  std::lock_guard<std::mutex> g(mu_);
  if (std::find(active_.begin(), active_.end(), request_id) == active_.end())
    active_.push_back(request_id);
}

bool BatchSchedulerCore::Complete(uint64_t request_id) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = std::find(active_.begin(), active_.end(), request_id);
  if (it == active_.end()) return false;
  active_.erase(it);
  return true;
}

bool BatchSchedulerCore::HasCapacity() const {
  std::lock_guard<std::mutex> g(mu_);
  return int64_t(active_.size()) < max_batch_;
}

std::vector<uint64_t> BatchSchedulerCore::Active() const {
  std::lock_guard<std::mutex> g(mu_);
  return active_;
}

int64_t BatchSchedulerCore::Queued() const {
  std::lock_guard<std::mutex> g(mu_);
  return int64_t(pending_.size());
}

int64_t BatchSchedulerCore::NumActive() const {
  std::lock_guard<std::mutex> g(mu_);
  return int64_t(active_.size());
}

void BatchSchedulerCore::WaitForWork(double timeout_s) {
  std::unique_lock<std::mutex> lk(mu_);
  if (!pending_.empty() || !active_.empty()) return;
  cv_.wait_for(lk, std::chrono::duration<double>(timeout_s),
               [&] { return !pending_.empty() || !active_.empty(); });
}

}  // namespace hcp::host
