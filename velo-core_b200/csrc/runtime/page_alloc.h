// page_alloc.h -- the KV page allocator (host side, no device work).
//
// Follows PagedAttentionBlockManager (src/paged_attention.rs:92-211): a FIFO
// of free page ids filled 0..total-1, `allocate(handle, token_len)` takes
// ceil(token_len / block_size) ids from the front (OutOfPages { requested,
// available } when short, nothing taken), `release(handle)` appends the
// handle's ids to the back (UnknownHandle when absent).  Allocating a handle
// that already holds pages replaces its mapping and the old ids are not
// returned to the pool (a BTreeMap insert over the old entry, :184).
#pragma once
#include <cstddef>
#include <cstdint>
#include <deque>
#include <map>
#include <vector>

namespace velo {

class PageAllocator {
public:
    PageAllocator(size_t block_size, size_t total_pages);

    size_t block_size() const { return block_size_; }
    size_t total_pages() const { return total_; }
    size_t free_pages() const { return free_.size(); }
    // pages_for_tokens (:150-152)
    size_t pages_for_tokens(size_t token_len) const {
        return token_len / block_size_ + (token_len % block_size_ != 0);
    }

    // 0, or VELO_ERR_OUT_OF_PAGES with *requested / *available set (state
    // unchanged).  The handle's ids, in allocation order, land in `pages`.
    int32_t allocate(uint64_t handle, size_t token_len, std::vector<uint32_t>* pages, size_t* requested,
                     size_t* available);
    // 0, or VELO_ERR_UNKNOWN_HANDLE
    int32_t release(uint64_t handle);
    // mapped_pages (:145-147): nullptr when the handle holds nothing
    const std::vector<uint32_t>* mapped(uint64_t handle) const;

private:
    size_t block_size_, total_;
    std::deque<uint32_t> free_;
    std::map<uint64_t, std::vector<uint32_t>> maps_;
};

}  // namespace velo
