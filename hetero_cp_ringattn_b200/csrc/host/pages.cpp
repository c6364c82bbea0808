// Page allocator of the paged KV arena.
//
// The device arena of a rank is [layers][pages][2][Hkv][page][D] (owned by the domain runtime);
// this allocator hands out page ids to requests and takes them back. Pages never move, so a
// request's page table stays valid for its whole life; running out raises a capacity error
// instead of growing with a copy (the reference's reserved slabs, self_driving.rs:146-331).
#include "hcp_host.h"

namespace hcp::host {

PageAllocator::PageAllocator(int64_t num_pages, int64_t page_size)
    : num_pages_(num_pages), page_size_(page_size) {
  if (num_pages < 0 || page_size <= 0) throw CapacityError("KV arena geometry must be positive");
  free_.reserve(size_t(num_pages));
  for (int64_t p = num_pages - 1; p >= 0; --p) free_.push_back(p);
}

std::vector<int64_t> PageAllocator::Alloc(int64_t n, int64_t request_id) {
  if (n < 0) throw CapacityError("negative page count");
  if (n > int64_t(free_.size()))
    throw CapacityError("KV arena out of pages: need " + std::to_string(n) + ", " +
                        std::to_string(free_.size()) + " free of " + std::to_string(num_pages_));
  std::vector<int64_t> out;
  out.reserve(size_t(n));
  for (int64_t k = 0; k < n; ++k) {
    const int64_t p = free_.back();
    free_.pop_back();
    owner_[p] = request_id;
    out.push_back(p);
  }
  return out;
}

void PageAllocator::Free(const std::vector<int64_t>& pages) {
  for (int64_t p : pages) {
    auto it = owner_.find(p);
    if (it == owner_.end()) continue;  // never handed out, or already free: nothing to return
    owner_.erase(it);
    free_.push_back(p);
  }
}

int64_t PageAllocator::OwnerOf(int64_t page) const {
  auto it = owner_.find(page);
  return it == owner_.end() ? -1 : it->second;
}

}  // namespace hcp::host
