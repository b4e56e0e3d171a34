// Host-side block bookkeeping of the paged KV cache, in C++: the free list, reference
// counts, the LRU set of evictable cached blocks, the content-hash -> block map and the
// per-sequence block tables. Semantics follow pagellm cache/paged.py:47-274
// (BlockAllocator, BlockManager); hashing itself (SHA-256 chains, plan_prefix,
// mark_computed's hash loop) stays with the Python caller, which hands digests in.
//
// Data structures: the free list is a ring buffer of capacity num_blocks (FIFO: allocate
// takes the oldest, decref returns to the back); the evictable set is an intrusive
// doubly-linked list over block ids in release order, so allocate evicts the
// least-recently released cached block in O(1) and incref revives any block in O(1).

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "pagekv.h"

namespace {

thread_local std::string g_bm_err;

int bm_fail(int code, const char* fmt, ...) {
    char buf[256];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_bm_err = buf;
    return code;
}

struct SeqTable {
    std::vector<int32_t> blocks;
    std::vector<std::string> hashes;  // digests of the leading full blocks (prefix chain)
};

}  // namespace

struct pk_block_manager {
    int64_t num_blocks = 0;
    int block_size = 0;
    bool prefix_caching = true;
    std::vector<int64_t> ref;
    // free list ring
    std::vector<int32_t> ring;
    int64_t head = 0, count = 0;
    // evictable LRU (intrusive list; -1 terminated)
    std::vector<int32_t> prev, next;
    std::vector<uint8_t> in_lru;
    int32_t lru_head = -1, lru_tail = -1;
    int64_t lru_count = 0;
    // prefix cache
    std::vector<std::string> hash_of;
    std::vector<uint8_t> has_hash;
    std::unordered_map<std::string, int32_t> cached;
    int64_t prefix_hits = 0, prefix_queries = 0;
    // tables
    std::unordered_map<int64_t, SeqTable> tables;

    int64_t num_free() const { return count + lru_count; }
    int64_t blocks_needed(int64_t tokens) const { return (tokens + block_size - 1) / block_size; }

    void free_push(int32_t b) {
        ring[(head + count) % num_blocks] = b;
        ++count;
    }
    int32_t free_pop() {
        int32_t b = ring[head];
        head = (head + 1) % num_blocks;
        --count;
        return b;
    }
    void lru_push(int32_t b) {
        prev[b] = lru_tail;
        next[b] = -1;
        if (lru_tail >= 0) next[lru_tail] = b; else lru_head = b;
        lru_tail = b;
        in_lru[b] = 1;
        ++lru_count;
    }
    void lru_remove(int32_t b) {
        if (prev[b] >= 0) next[prev[b]] = next[b]; else lru_head = next[b];
        if (next[b] >= 0) prev[next[b]] = prev[b]; else lru_tail = prev[b];
        prev[b] = next[b] = -1;
        in_lru[b] = 0;
        --lru_count;
    }

    int allocate(int32_t* out) {
        int32_t b;
        if (count > 0) {
            b = free_pop();
        } else if (lru_count > 0) {
            b = lru_head;
            lru_remove(b);
            cached.erase(hash_of[b]);
            hash_of[b].clear();
            has_hash[b] = 0;
        } else {
            return bm_fail(PK_ERR_OUT_OF_BLOCKS, "KV cache is full");
        }
        if (ref[b] != 0) return bm_fail(PK_ERR_INVALID_ARG, "internal: allocated block %d has ref %lld", b, (long long)ref[b]);
        ref[b] = 1;
        *out = b;
        return PK_OK;
    }
    int check_id(int64_t b) const {
        if (b < 0 || b >= num_blocks)
            return bm_fail(PK_ERR_OUT_OF_RANGE, "block id %lld outside [0, %lld)", (long long)b, (long long)num_blocks);
        return PK_OK;
    }
    int incref(int32_t b) {
        int rc = check_id(b);
        if (rc) return rc;
        if (ref[b] == 0) {
            if (!in_lru[b]) return bm_fail(PK_ERR_NOT_FOUND, "block %d is neither referenced nor cached", b);
            lru_remove(b);
        }
        ++ref[b];
        return PK_OK;
    }
    int decref(int32_t b) {
        int rc = check_id(b);
        if (rc) return rc;
        if (ref[b] <= 0) return bm_fail(PK_ERR_DOUBLE_FREE, "double free of block %d", b);
        if (--ref[b] == 0) {
            if (has_hash[b]) lru_push(b); else free_push(b);
        }
        return PK_OK;
    }
    void reg(int32_t b, const std::string& h) {
        if (!prefix_caching || has_hash[b] || cached.count(h)) return;
        cached.emplace(h, b);
        hash_of[b] = h;
        has_hash[b] = 1;
    }
};

namespace {

int get_table(pk_block_manager* m, int64_t seq, SeqTable** t) {
    auto it = m->tables.find(seq);
    if (it == m->tables.end()) return bm_fail(PK_ERR_NOT_FOUND, "unknown sequence %lld", (long long)seq);
    *t = &it->second;
    return PK_OK;
}

int copy_out(const std::vector<int32_t>& v, int32_t* out, int64_t cap, int64_t* n) {
    if (n) *n = static_cast<int64_t>(v.size());
    if (out && cap < static_cast<int64_t>(v.size()))
        return bm_fail(PK_ERR_INVALID_ARG, "output buffer holds %lld, need %zu", (long long)cap, v.size());
    if (out && !v.empty()) std::memcpy(out, v.data(), v.size() * sizeof(int32_t));
    return PK_OK;
}

}  // namespace

extern "C" {

PK_API const char* pk_bm_last_error(void) { return g_bm_err.c_str(); }

PK_API int pk_bm_create(int64_t num_blocks, int block_size, int enable_prefix_caching,
                        pk_block_manager** out) {
    if (!out) return bm_fail(PK_ERR_INVALID_ARG, "out is NULL");
    if (num_blocks < 0 || num_blocks >= (int64_t(1) << 31) || block_size <= 0)
        return bm_fail(PK_ERR_INVALID_ARG, "num_blocks must be in [0, 2^31), block_size > 0");
    auto* m = new pk_block_manager();
    m->num_blocks = num_blocks;
    m->block_size = block_size;
    m->prefix_caching = enable_prefix_caching != 0;
    m->ref.assign(num_blocks, 0);
    m->ring.resize(num_blocks);
    for (int64_t b = 0; b < num_blocks; ++b) m->ring[b] = static_cast<int32_t>(b);
    m->count = num_blocks;
    m->prev.assign(num_blocks, -1);
    m->next.assign(num_blocks, -1);
    m->in_lru.assign(num_blocks, 0);
    m->hash_of.resize(num_blocks);
    m->has_hash.assign(num_blocks, 0);
    *out = m;
    return PK_OK;
}

PK_API int pk_bm_destroy(pk_block_manager* m) {
    delete m;
    return PK_OK;
}

// ---------------------------------------------------------------- BlockAllocator
PK_API int pk_bm_allocate_block(pk_block_manager* m, int32_t* block) {
    if (!m || !block) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    return m->allocate(block);
}

PK_API int pk_bm_incref(pk_block_manager* m, int32_t block) {
    if (!m) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    return m->incref(block);
}

PK_API int pk_bm_decref(pk_block_manager* m, int32_t block) {
    if (!m) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    return m->decref(block);
}

PK_API int pk_bm_lookup(pk_block_manager* m, const uint8_t* hash, int64_t len, int32_t* block) {
    if (!m || !block || (len > 0 && !hash)) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    *block = -1;
    if (!m->prefix_caching) return PK_OK;
    auto it = m->cached.find(std::string(reinterpret_cast<const char*>(hash), static_cast<size_t>(len)));
    if (it != m->cached.end()) *block = it->second;
    return PK_OK;
}

PK_API int pk_bm_register(pk_block_manager* m, int32_t block, const uint8_t* hash, int64_t len) {
    if (!m || (len > 0 && !hash)) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    int rc = m->check_id(block);
    if (rc) return rc;
    m->reg(block, std::string(reinterpret_cast<const char*>(hash), static_cast<size_t>(len)));
    return PK_OK;
}

// counts[0] num_free, [1] free-list length, [2] evictable, [3] cached hashes,
// [4] prefix_hits, [5] prefix_queries, [6] sequences
PK_API int pk_bm_counts(const pk_block_manager* m, int64_t* c7) {
    if (!m || !c7) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    c7[0] = m->num_free();
    c7[1] = m->count;
    c7[2] = m->lru_count;
    c7[3] = static_cast<int64_t>(m->cached.size());
    c7[4] = m->prefix_hits;
    c7[5] = m->prefix_queries;
    c7[6] = static_cast<int64_t>(m->tables.size());
    return PK_OK;
}

// Live pointer to the int64 ref-count array (valid for the manager's lifetime).
PK_API int pk_bm_refcounts(pk_block_manager* m, int64_t** ref) {
    if (!m || !ref) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    *ref = m->ref.data();
    return PK_OK;
}

PK_API int pk_bm_free_list(const pk_block_manager* m, int32_t* out, int64_t cap, int64_t* n) {
    if (!m) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    std::vector<int32_t> v;
    v.reserve(m->count);
    for (int64_t i = 0; i < m->count; ++i) v.push_back(m->ring[(m->head + i) % m->num_blocks]);
    return copy_out(v, out, cap, n);
}

PK_API int pk_bm_evictable_list(const pk_block_manager* m, int32_t* out, int64_t cap, int64_t* n) {
    if (!m) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    std::vector<int32_t> v;
    for (int32_t b = m->lru_head; b >= 0; b = m->next[b]) v.push_back(b);
    return copy_out(v, out, cap, n);
}

// The content hash a block is published under: *len = -1 if none, else its length, and the
// bytes are copied to out when cap allows.
PK_API int pk_bm_block_hash(const pk_block_manager* m, int32_t block, uint8_t* out, int64_t cap,
                            int64_t* len) {
    if (!m || !len) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    int rc = m->check_id(block);
    if (rc) return rc;
    if (!m->has_hash[block]) {
        *len = -1;
        return PK_OK;
    }
    const std::string& h = m->hash_of[block];
    *len = static_cast<int64_t>(h.size());
    if (out && cap >= *len) std::memcpy(out, h.data(), h.size());
    return PK_OK;
}

PK_API int pk_bm_add_prefix_stats(pk_block_manager* m, int64_t hits, int64_t queries) {
    if (!m) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    m->prefix_hits += hits;
    m->prefix_queries += queries;
    return PK_OK;
}

// ---------------------------------------------------------------- BlockManager
// allocate (paged.py:187-203) after the caller's plan_prefix: hit blocks are increfed in
// order, then the remaining blocks_needed(n_tokens) - n_hits are allocated fresh. The hit
// digests become the sequence's hash chain (concatenated, hash_len bytes each).
// Returns the number of cached tokens in *cached_tokens.
PK_API int pk_bm_seq_allocate(pk_block_manager* m, int64_t seq, int64_t n_tokens,
                              const int32_t* hits, int64_t n_hits, const uint8_t* hashes,
                              int64_t hash_len, int64_t* cached_tokens) {
    if (!m || (n_hits > 0 && !hits)) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    if (m->tables.count(seq)) return bm_fail(PK_ERR_DUPLICATE, "seq %lld already has blocks", (long long)seq);
    int64_t revived = 0;
    for (int64_t i = 0; i < n_hits; ++i) {
        int rc = m->check_id(hits[i]);
        if (rc) return rc;
        if (m->ref[hits[i]] == 0) ++revived;
    }
    const int64_t need = m->blocks_needed(n_tokens) - n_hits + revived;
    if (need > m->num_free()) return bm_fail(PK_ERR_OUT_OF_BLOCKS, "not enough blocks for prompt");
    // Python floor division, as pagellm counts it: an empty prompt counts -1.
    const int64_t q = n_tokens - 1;
    m->prefix_queries += q >= 0 ? q / m->block_size : -((-q + m->block_size - 1) / m->block_size);
    m->prefix_hits += n_hits;
    SeqTable t;
    for (int64_t i = 0; i < n_hits; ++i) {
        int rc = m->incref(hits[i]);
        if (rc) return rc;
        t.blocks.push_back(hits[i]);
        t.hashes.emplace_back(reinterpret_cast<const char*>(hashes) + i * hash_len,
                              static_cast<size_t>(hash_len));
    }
    const int64_t fresh = m->blocks_needed(n_tokens) - n_hits;
    for (int64_t i = 0; i < fresh; ++i) {
        int32_t b;
        int rc = m->allocate(&b);
        if (rc) return rc;
        t.blocks.push_back(b);
    }
    m->tables.emplace(seq, std::move(t));
    if (cached_tokens) *cached_tokens = n_hits * m->block_size;
    return PK_OK;
}

// can_append (paged.py:206-213)
PK_API int pk_bm_can_append(pk_block_manager* m, int64_t seq, int64_t n_tokens, int* ok) {
    if (!m || !ok) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    SeqTable* t;
    int rc = get_table(m, seq, &t);
    if (rc) return rc;
    int64_t need = m->blocks_needed(n_tokens) - static_cast<int64_t>(t->blocks.size());
    if (!t->blocks.empty() && m->ref[t->blocks.back()] > 1) ++need;
    *ok = need <= m->num_free();
    return PK_OK;
}

// ensure_capacity (paged.py:215-239): privatise the shared blocks from write_from on and
// grow to n_tokens. Writes up to cap (src, dst) pairs to pairs_out; *npairs = count.
PK_API int pk_bm_ensure_capacity(pk_block_manager* m, int64_t seq, int64_t n_tokens,
                                 int64_t write_from, int64_t* pairs_out, int64_t cap,
                                 int64_t* npairs) {
    if (!m || !npairs) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    if (write_from < 0) return bm_fail(PK_ERR_INVALID_ARG, "write_from < 0");
    SeqTable* t;
    int rc = get_table(m, seq, &t);
    if (rc) return rc;
    std::vector<int64_t> pairs;
    const int64_t first = write_from / m->block_size;
    for (int64_t i = first; i < static_cast<int64_t>(t->blocks.size()); ++i) {
        const int32_t b = t->blocks[i];
        if (m->ref[b] > 1) {
            int32_t nb;
            rc = m->allocate(&nb);
            if (rc) return rc;
            rc = m->decref(b);
            if (rc) return rc;
            t->blocks[i] = nb;
            pairs.push_back(b);
            pairs.push_back(nb);
            if (static_cast<int64_t>(t->hashes.size()) > i) t->hashes.resize(i);
        }
    }
    while (static_cast<int64_t>(t->blocks.size()) < m->blocks_needed(n_tokens)) {
        int32_t nb;
        rc = m->allocate(&nb);
        if (rc) return rc;
        t->blocks.push_back(nb);
    }
    *npairs = static_cast<int64_t>(pairs.size() / 2);
    if (pairs_out) {
        if (cap < *npairs) return bm_fail(PK_ERR_INVALID_ARG, "pairs buffer too small");
        std::memcpy(pairs_out, pairs.data(), pairs.size() * sizeof(int64_t));
    }
    return PK_OK;
}

// Hash chain length of a sequence and (optionally) its last digest.
PK_API int pk_bm_seq_hashes(pk_block_manager* m, int64_t seq, int64_t* n, uint8_t* last,
                            int64_t cap, int64_t* last_len) {
    if (!m || !n) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    SeqTable* t;
    int rc = get_table(m, seq, &t);
    if (rc) return rc;
    *n = static_cast<int64_t>(t->hashes.size());
    if (last_len) *last_len = t->hashes.empty() ? -1 : static_cast<int64_t>(t->hashes.back().size());
    if (last && !t->hashes.empty() && cap >= static_cast<int64_t>(t->hashes.back().size()))
        std::memcpy(last, t->hashes.back().data(), t->hashes.back().size());
    return PK_OK;
}

// Digest at position i of a sequence's hash chain (*len = its length).
PK_API int pk_bm_seq_hash_at(pk_block_manager* m, int64_t seq, int64_t i, uint8_t* out, int64_t cap,
                             int64_t* len) {
    if (!m || !len) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    SeqTable* t;
    int rc = get_table(m, seq, &t);
    if (rc) return rc;
    if (i < 0 || i >= static_cast<int64_t>(t->hashes.size())) return bm_fail(PK_ERR_OUT_OF_RANGE, "hash index");
    *len = static_cast<int64_t>(t->hashes[i].size());
    if (out && cap >= *len) std::memcpy(out, t->hashes[i].data(), t->hashes[i].size());
    return PK_OK;
}

// mark_computed's bookkeeping half (paged.py:241-254): append `count` digests to the
// sequence's chain and publish block i (chain position i) under each.
PK_API int pk_bm_seq_push_hashes(pk_block_manager* m, int64_t seq, const uint8_t* hashes,
                                 int64_t hash_len, int64_t count) {
    if (!m || (count > 0 && !hashes)) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    SeqTable* t;
    int rc = get_table(m, seq, &t);
    if (rc) return rc;
    for (int64_t k = 0; k < count; ++k) {
        const size_t i = t->hashes.size();
        if (i >= t->blocks.size()) return bm_fail(PK_ERR_OUT_OF_RANGE, "hash chain longer than the table");
        t->hashes.emplace_back(reinterpret_cast<const char*>(hashes) + k * hash_len,
                               static_cast<size_t>(hash_len));
        m->reg(t->blocks[i], t->hashes.back());
    }
    return PK_OK;
}

// fork (paged.py:257-263): child shares every parent block (replacing any child table).
PK_API int pk_bm_fork(pk_block_manager* m, int64_t parent, int64_t child) {
    if (!m) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    SeqTable* p;
    int rc = get_table(m, parent, &p);
    if (rc) return rc;
    for (int32_t b : p->blocks) {
        rc = m->incref(b);
        if (rc) return rc;
    }
    SeqTable c = *p;
    m->tables[child] = std::move(c);
    return PK_OK;
}

// free (paged.py:265-271): drop the table, releasing blocks tail first.
PK_API int pk_bm_free_seq(pk_block_manager* m, int64_t seq) {
    if (!m) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    auto it = m->tables.find(seq);
    if (it == m->tables.end()) return bm_fail(PK_ERR_NOT_FOUND, "unknown sequence %lld", (long long)seq);
    std::vector<int32_t> blocks = std::move(it->second.blocks);
    m->tables.erase(it);
    for (auto b = blocks.rbegin(); b != blocks.rend(); ++b) {
        int rc = m->decref(*b);
        if (rc) return rc;
    }
    return PK_OK;
}

// Paged speculative rollback: keep the first n_tokens of a sequence. pagellm rolls back only
// contiguous caches (cache/contiguous.py:33-38, engine/speculative.py:136-137; paged rollback
// is on its roadmap, README.md:370); this is its paged form. Blocks past the kept tokens are
// released last block first, as free does (paged.py:265-271); the hash chain keeps only the
// full blocks that remain; a kept partial last block that is published in the prefix cache
// and held by this sequence alone is unpublished, since the next writes change it in place
// (a shared one is copied on write by ensure_capacity instead, so its content stays).
PK_API int pk_bm_truncate(pk_block_manager* m, int64_t seq, int64_t n_tokens) {
    if (!m) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    SeqTable* t;
    int rc = get_table(m, seq, &t);
    if (rc) return rc;
    const int64_t cap = static_cast<int64_t>(t->blocks.size()) * m->block_size;
    if (n_tokens < 0 || n_tokens > cap)
        return bm_fail(PK_ERR_INVALID_ARG, "cannot truncate a %lld-token table to %lld tokens", (long long)cap,
                       (long long)n_tokens);
    const int64_t keep = m->blocks_needed(n_tokens), full = n_tokens / m->block_size;
    while (static_cast<int64_t>(t->blocks.size()) > keep) {
        const int32_t b = t->blocks.back();
        t->blocks.pop_back();
        rc = m->decref(b);
        if (rc) return rc;
    }
    if (static_cast<int64_t>(t->hashes.size()) > full) t->hashes.resize(full);
    if (keep > full) {
        const int32_t b = t->blocks[full];
        if (m->ref[b] == 1 && m->has_hash[b]) {
            m->cached.erase(m->hash_of[b]);
            m->hash_of[b].clear();
            m->has_hash[b] = 0;
        }
    }
    return PK_OK;
}

PK_API int pk_bm_table(const pk_block_manager* m, int64_t seq, int32_t* out, int64_t cap, int64_t* n) {
    if (!m) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    auto it = m->tables.find(seq);
    if (it == m->tables.end()) return bm_fail(PK_ERR_NOT_FOUND, "unknown sequence %lld", (long long)seq);
    return copy_out(it->second.blocks, out, cap, n);
}

PK_API int pk_bm_seq_ids(const pk_block_manager* m, int64_t* out, int64_t cap, int64_t* n) {
    if (!m || !n) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    *n = static_cast<int64_t>(m->tables.size());
    if (out) {
        if (cap < *n) return bm_fail(PK_ERR_INVALID_ARG, "buffer too small");
        int64_t i = 0;
        for (const auto& kv : m->tables) out[i++] = kv.first;
    }
    return PK_OK;
}

// Block tables of `nseq` sequences in CSR form (the input pk_batch_plan takes), built
// without a round trip through Python lists. indptr has nseq+1 entries; ids needs
// *total entries (call with ids = NULL to size it).
PK_API int pk_bm_tables_csr(const pk_block_manager* m, const int64_t* seqs, int64_t nseq,
                            int64_t* indptr, int32_t* ids, int64_t cap, int64_t* total) {
    if (!m || !total || (nseq > 0 && !seqs)) return bm_fail(PK_ERR_INVALID_ARG, "NULL pointer");
    int64_t acc = 0;
    if (indptr) indptr[0] = 0;
    for (int64_t i = 0; i < nseq; ++i) {
        auto it = m->tables.find(seqs[i]);
        if (it == m->tables.end()) return bm_fail(PK_ERR_NOT_FOUND, "unknown sequence %lld", (long long)seqs[i]);
        const auto& b = it->second.blocks;
        if (ids) {
            if (acc + static_cast<int64_t>(b.size()) > cap) return bm_fail(PK_ERR_INVALID_ARG, "ids buffer too small");
            if (!b.empty()) std::memcpy(ids + acc, b.data(), b.size() * sizeof(int32_t));
        }
        acc += static_cast<int64_t>(b.size());
        if (indptr) indptr[i + 1] = acc;
    }
    *total = acc;
    return PK_OK;
}

}  // extern "C"
