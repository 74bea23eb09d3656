// shard.cpp -- tensor-parallel weight sharding on the host (C ABI,
// include/velo_cuda.h), following src/metal/sharding.rs:28-126: q, k, v, w1,
// w3 and the LM head are split by output rows (Column), wo and w2 by input
// columns (Row, on q4_0 block boundaries), everything else is replicated.
#include <cstring>

#include "runtime/context.h"
#include "runtime/shard.h"

namespace velo {

int32_t shard_strategy(const char* name) {
    const std::string n = name ? name : "";
    auto has = [&](const char* s) { return n.find(s) != std::string::npos; };
    if (has("attention.wq") || has("attention.wk") || has("attention.wv")) return VELO_SHARD_COLUMN;
    if (has("attention.wo")) return VELO_SHARD_ROW;
    if (has("feed_forward.w1") || has("feed_forward.w3")) return VELO_SHARD_COLUMN;
    if (has("feed_forward.w2")) return VELO_SHARD_ROW;
    if (n == "output.weight") return VELO_SHARD_COLUMN;
    return VELO_SHARD_REPLICATED;
}

static size_t dtype_row_bytes(int dt, uint64_t cols) {
    return dt == VELO_DT_F32 ? cols * 4 : dt == VELO_DT_F16 ? cols * 2 : cols / 32 * 18;
}

int32_t shard_weight(const velo_weight_desc& w, int32_t strategy, int tp, int rank,
                     std::vector<uint8_t>& out, uint64_t& rows_out, uint64_t& cols_out) {
    const size_t rb = dtype_row_bytes(w.dtype, w.cols);
    const uint8_t* src = static_cast<const uint8_t*>(w.data);
    if (tp <= 1 || strategy == VELO_SHARD_REPLICATED) {
        out.assign(src, src + rb * w.rows);
        rows_out = w.rows;
        cols_out = w.cols;
        return VELO_OK;
    }
    if (strategy == VELO_SHARD_COLUMN) {
        if (w.rows % tp)
            return fail(VELO_ERR_INVALID_ARGUMENT, "Tensor %s rows (%llu) not divisible by TP degree %d",
                        w.name ? w.name : "?", (unsigned long long)w.rows, tp);
        const uint64_t sr = w.rows / tp;
        out.assign(src + rank * sr * rb, src + (rank + 1) * sr * rb);
        rows_out = sr;
        cols_out = w.cols;
        return VELO_OK;
    }
    if (strategy == VELO_SHARD_ROW) {
        if (w.cols % tp)
            return fail(VELO_ERR_INVALID_ARGUMENT, "Tensor %s cols (%llu) not divisible by TP degree %d",
                        w.name ? w.name : "?", (unsigned long long)w.cols, tp);
        const uint64_t sc = w.cols / tp;
        const uint64_t block = w.dtype == VELO_DT_Q4_0 ? 32 : 1;
        if (sc % block)
            return fail(VELO_ERR_INVALID_ARGUMENT, "Tensor %s shard cols (%llu) must be multiple of block size %llu",
                        w.name ? w.name : "?", (unsigned long long)sc, (unsigned long long)block);
        const size_t srb = rb / tp;
        out.resize(srb * w.rows);
        for (uint64_t r = 0; r < w.rows; ++r) std::memcpy(out.data() + r * srb, src + r * rb + rank * srb, srb);
        rows_out = w.rows;
        cols_out = sc;
        return VELO_OK;
    }
    return fail(VELO_ERR_INVALID_ARGUMENT, "unknown shard strategy %d", strategy);
}

}  // namespace velo

using velo::fail;

extern "C" {

int32_t velo_cuda_shard_strategy(const char* name) { return velo::shard_strategy(name); }

int32_t velo_cuda_shard_weight(const velo_weight_desc* w, int32_t strategy, int32_t tp, int32_t rank,
                               void* out, size_t out_bytes, uint64_t* out_rows, uint64_t* out_cols) {
    velo::clear_last_error();
    if (!w || !w->data || !out_rows || !out_cols) return fail(VELO_ERR_INVALID_ARGUMENT, "NULL argument");
    if (tp < 1 || rank < 0 || rank >= tp) return fail(VELO_ERR_INVALID_ARGUMENT, "rank %d of %d", rank, tp);
    if (w->dtype < VELO_DT_F32 || w->dtype > VELO_DT_Q4_0 || (w->dtype == VELO_DT_Q4_0 && w->cols % 32))
        return fail(VELO_ERR_INVALID_ARGUMENT, "tensor %s: bad dtype", w->name ? w->name : "?");
    std::vector<uint8_t> buf;
    uint64_t r = 0, c = 0;
    int32_t st = velo::shard_weight(*w, strategy, tp, rank, buf, r, c);
    if (st) return st;
    if (!out || out_bytes < buf.size())
        return fail(VELO_ERR_INVALID_ARGUMENT, "output buffer of %zu bytes, need %zu", out_bytes, buf.size());
    std::memcpy(out, buf.data(), buf.size());
    *out_rows = r;
    *out_cols = c;
    return VELO_OK;
}

}  // extern "C"
