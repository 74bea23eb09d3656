// page_alloc.cpp -- KV page allocator and its host-only C ABI
// (include/velo_cuda.h, velo_page_allocator_*), following
// PagedAttentionBlockManager (src/paged_attention.rs:92-211).
#include "runtime/page_alloc.h"

#include "runtime/context.h"

namespace velo {

PageAllocator::PageAllocator(size_t block_size, size_t total_pages)
    : block_size_(block_size), total_(total_pages) {
    for (size_t i = 0; i < total_pages; ++i) free_.push_back((uint32_t)i);
}

int32_t PageAllocator::allocate(uint64_t handle, size_t token_len, std::vector<uint32_t>* pages,
                                size_t* requested, size_t* available) {
    const size_t req = pages_for_tokens(token_len);
    if (req > free_.size()) {
        if (requested) *requested = req;
        if (available) *available = free_.size();
        return VELO_ERR_OUT_OF_PAGES;
    }
    std::vector<uint32_t> got(free_.begin(), free_.begin() + (std::ptrdiff_t)req);
    free_.erase(free_.begin(), free_.begin() + (std::ptrdiff_t)req);
    if (pages) *pages = got;
    maps_[handle] = std::move(got);  // replaces an existing mapping
    return VELO_OK;
}

int32_t PageAllocator::release(uint64_t handle) {
    auto it = maps_.find(handle);
    if (it == maps_.end()) return VELO_ERR_UNKNOWN_HANDLE;
    for (uint32_t p : it->second) free_.push_back(p);
    maps_.erase(it);
    return VELO_OK;
}

const std::vector<uint32_t>* PageAllocator::mapped(uint64_t handle) const {
    auto it = maps_.find(handle);
    return it == maps_.end() ? nullptr : &it->second;
}

}  // namespace velo

struct velo_page_allocator {
    velo::PageAllocator a;
    velo_page_allocator(size_t bs, size_t total) : a(bs, total) {}
};

using velo::fail;

extern "C" {

int32_t velo_page_allocator_create(size_t block_size, size_t total_pages, velo_page_allocator** out) {
    velo::clear_last_error();
    if (!out) return fail(VELO_ERR_INVALID_ARGUMENT, "out is NULL");
    *out = nullptr;
    if (block_size == 0) return fail(VELO_ERR_INVALID_BLOCK_SIZE, "InvalidBlockSize");
    if (total_pages > 0xffffffffull)
        return fail(VELO_ERR_INVALID_ARGUMENT, "total_pages %zu does not fit 32-bit page ids", total_pages);
    *out = new velo_page_allocator(block_size, total_pages);
    return VELO_OK;
}

void velo_page_allocator_destroy(velo_page_allocator* a) { delete a; }

int32_t velo_page_allocator_allocate(velo_page_allocator* a, uint64_t handle, size_t token_len,
                                     uint32_t* pages_out, size_t pages_cap, size_t* n_pages,
                                     size_t* requested, size_t* available) {
    velo::clear_last_error();
    if (!a) return fail(VELO_ERR_INVALID_ARGUMENT, "allocator is NULL");
    const size_t req = a->a.pages_for_tokens(token_len);
    if (pages_out && pages_cap < req && req <= a->a.free_pages())
        return fail(VELO_ERR_INVALID_ARGUMENT, "pages_out holds %zu ids, %zu needed", pages_cap, req);
    std::vector<uint32_t> got;
    size_t rq = 0, av = 0;
    const int32_t st = a->a.allocate(handle, token_len, &got, &rq, &av);
    if (requested) *requested = st ? rq : req;
    if (available) *available = st ? av : a->a.free_pages();
    if (st) return fail(st, "OutOfPages { requested: %zu, available: %zu }", rq, av);
    if (n_pages) *n_pages = got.size();
    if (pages_out)
        for (size_t i = 0; i < got.size(); ++i) pages_out[i] = got[i];
    return VELO_OK;
}

int32_t velo_page_allocator_release(velo_page_allocator* a, uint64_t handle) {
    velo::clear_last_error();
    if (!a) return fail(VELO_ERR_INVALID_ARGUMENT, "allocator is NULL");
    const int32_t st = a->a.release(handle);
    if (st) return fail(st, "UnknownHandle(%llu)", (unsigned long long)handle);
    return VELO_OK;
}

int32_t velo_page_allocator_mapped_pages(const velo_page_allocator* a, uint64_t handle, uint32_t* pages_out,
                                         size_t pages_cap, size_t* n_pages) {
    velo::clear_last_error();
    if (!a) return fail(VELO_ERR_INVALID_ARGUMENT, "allocator is NULL");
    const std::vector<uint32_t>* m = a->a.mapped(handle);
    if (!m) return fail(VELO_ERR_UNKNOWN_HANDLE, "UnknownHandle(%llu)", (unsigned long long)handle);
    if (n_pages) *n_pages = m->size();
    if (pages_out) {
        if (pages_cap < m->size())
            return fail(VELO_ERR_INVALID_ARGUMENT, "pages_out holds %zu ids, %zu mapped", pages_cap, m->size());
        for (size_t i = 0; i < m->size(); ++i) pages_out[i] = (*m)[i];
    }
    return VELO_OK;
}

size_t velo_page_allocator_free_pages(const velo_page_allocator* a) { return a ? a->a.free_pages() : 0; }

size_t velo_page_allocator_pages_for_tokens(const velo_page_allocator* a, size_t token_len) {
    return a ? a->a.pages_for_tokens(token_len) : 0;
}

}  // extern "C"
