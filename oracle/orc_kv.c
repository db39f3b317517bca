/*
 * orc_kv.c -- oracle for the paged-KV block tables and the draft-tree shape.
 * TEST INFRASTRUCTURE ONLY.
 *
 * The table logic restates PagedKVCache (server/paged_kv_cache.cpp):
 *   append_tokens          :50-102  lowest-free-index linear scan (68-77),
 *                                   OOM stops the append (78-81)
 *   free_request           :123-134
 *   share_prefix           :136-154 (overwrites an existing table of new_req
 *                                   without releasing it, as the reference does)
 *   free_merged_blocks     :178-194 (length drops by n*block_size)
 *   evict_least_important  :207-228 (whole tail blocks until >= n tokens)
 *   get_utilization        :197-204
 * plus the token-granular truncate used to roll back rejected draft slots.
 */
#include "oracle.h"

#include <stdlib.h>
#include <string.h>

struct orc_blockmgr {
    int num_blocks, block_size, max_reqs, max_bpr;
    int* ref;
    int* nblk;   /* -1 = no table */
    int* len;
    int* tab;    /* [max_reqs, max_bpr] */
};

orc_blockmgr* orc_bm_create(int num_blocks, int block_size, int max_reqs, int max_blocks_per_req) {
    orc_blockmgr* bm = (orc_blockmgr*)calloc(1, sizeof(orc_blockmgr));
    bm->num_blocks = num_blocks;
    bm->block_size = block_size;
    bm->max_reqs = max_reqs;
    bm->max_bpr = max_blocks_per_req;
    bm->ref = (int*)calloc(num_blocks, sizeof(int));
    bm->nblk = (int*)malloc(sizeof(int) * max_reqs);
    bm->len = (int*)calloc(max_reqs, sizeof(int));
    bm->tab = (int*)malloc(sizeof(int) * (size_t)max_reqs * max_blocks_per_req);
    for (int r = 0; r < max_reqs; ++r) bm->nblk[r] = -1;
    return bm;
}

void orc_bm_free(orc_blockmgr* bm) {
    if (!bm) return;
    free(bm->ref); free(bm->nblk); free(bm->len); free(bm->tab); free(bm);
}

static void ensure_table(orc_blockmgr* bm, int req) {
    if (bm->nblk[req] < 0) { bm->nblk[req] = 0; bm->len[req] = 0; }
}

int orc_bm_append(orc_blockmgr* bm, int req, int n_tokens) {
    ensure_table(bm, req);
    if (n_tokens <= 0) return -1;
    int last = -1, done = 0;
    while (done < n_tokens) {
        int off = bm->len[req] % bm->block_size;
        int cur = bm->len[req] / bm->block_size;
        if (cur >= bm->nblk[req]) {
            int fb = -1;
            for (int b = 0; b < bm->num_blocks; ++b)
                if (bm->ref[b] == 0) { fb = b; bm->ref[b] = 1; break; }
            if (fb < 0 || bm->nblk[req] >= bm->max_bpr) {
                if (fb >= 0) bm->ref[fb] = 0;
                break; /* OOM: stop the append */
            }
            bm->tab[(size_t)req * bm->max_bpr + bm->nblk[req]++] = fb;
        }
        int phys = bm->tab[(size_t)req * bm->max_bpr + cur];
        int n = bm->block_size - off;
        if (n > n_tokens - done) n = n_tokens - done;
        done += n;
        bm->len[req] += n;
        last = phys;
    }
    return last;
}

void orc_bm_free_request(orc_blockmgr* bm, int req) {
    if (bm->nblk[req] < 0) return;
    for (int i = 0; i < bm->nblk[req]; ++i) {
        int p = bm->tab[(size_t)req * bm->max_bpr + i];
        if (p >= 0 && p < bm->num_blocks) bm->ref[p]--;
    }
    bm->nblk[req] = -1;
    bm->len[req] = 0;
}

void orc_bm_share_prefix(orc_blockmgr* bm, int new_req, int src_req, int shared_len) {
    if (bm->nblk[src_req] < 0) return;
    int want = (shared_len + bm->block_size - 1) / bm->block_size;
    int n = 0;
    int tmp[4096];
    for (int i = 0; i < want && i < bm->nblk[src_req] && n < 4096; ++i) {
        int p = bm->tab[(size_t)src_req * bm->max_bpr + i];
        tmp[n++] = p;
        bm->ref[p]++;
    }
    bm->nblk[new_req] = n;
    bm->len[new_req] = shared_len;
    memcpy(bm->tab + (size_t)new_req * bm->max_bpr, tmp, sizeof(int) * n);
}

void orc_bm_free_tail_blocks(orc_blockmgr* bm, int req, int n_blocks) {
    if (bm->nblk[req] < 0 || n_blocks <= 0) return;
    int freed = 0;
    while (bm->nblk[req] > 0 && freed < n_blocks) {
        int p = bm->tab[(size_t)req * bm->max_bpr + --bm->nblk[req]];
        if (p >= 0 && p < bm->num_blocks) bm->ref[p]--;
        ++freed;
    }
    bm->len[req] -= n_blocks * bm->block_size;
    if (bm->len[req] < 0) bm->len[req] = 0;
}

int orc_bm_evict_tokens(orc_blockmgr* bm, int req, int n_tokens) {
    if (bm->nblk[req] < 0 || n_tokens <= 0) return 0;
    int freed = 0;
    while (bm->nblk[req] > 0 && freed < n_tokens) {
        int p = bm->tab[(size_t)req * bm->max_bpr + --bm->nblk[req]];
        if (p >= 0 && p < bm->num_blocks) bm->ref[p]--;
        freed += bm->block_size;
    }
    bm->len[req] -= freed;
    if (bm->len[req] < 0) bm->len[req] = 0;
    return 1;
}

void orc_bm_truncate(orc_blockmgr* bm, int req, int new_len) {
    if (bm->nblk[req] < 0) return;
    if (new_len < 0) new_len = 0;
    if (new_len > bm->len[req]) return;
    int keep = (new_len + bm->block_size - 1) / bm->block_size;
    while (bm->nblk[req] > keep) {
        int p = bm->tab[(size_t)req * bm->max_bpr + --bm->nblk[req]];
        if (p >= 0 && p < bm->num_blocks) bm->ref[p]--;
    }
    bm->len[req] = new_len;
}

float orc_bm_utilization(const orc_blockmgr* bm) {
    int used = 0;
    for (int b = 0; b < bm->num_blocks; ++b) used += bm->ref[b] > 0;
    return (float)used / (float)bm->num_blocks;
}

int orc_bm_table(const orc_blockmgr* bm, int req, int32_t* blocks, int cap, int32_t* len) {
    if (bm->nblk[req] < 0) { *len = 0; return 0; }
    int n = bm->nblk[req] < cap ? bm->nblk[req] : cap;
    for (int i = 0; i < n; ++i) blocks[i] = bm->tab[(size_t)req * bm->max_bpr + i];
    *len = bm->len[req];
    return bm->nblk[req];
}

int orc_bm_refcount(const orc_blockmgr* bm, int blk) { return bm->ref[blk]; }

int orc_tree_build(const int* branching, int levels, int max_nodes, int32_t* parent, int32_t* depth, int32_t* rank,
                   uint64_t* anc_mask) {
    int n = 1;
    parent[0] = -1; depth[0] = 0; rank[0] = 0; anc_mask[0] = 1ull;
    int lvl_begin = 0, lvl_end = 1;
    for (int L = 0; L < levels && n < max_nodes; ++L) {
        for (int p = lvl_begin; p < lvl_end && n < max_nodes; ++p)
            for (int c = 0; c < branching[L] && n < max_nodes; ++c) {
                parent[n] = p;
                depth[n] = depth[p] + 1;
                rank[n] = c;
                anc_mask[n] = anc_mask[p] | (1ull << n);
                ++n;
            }
        lvl_begin = lvl_end;
        lvl_end = n;
    }
    return n;
}
