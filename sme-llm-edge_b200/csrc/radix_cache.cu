// radix_cache.cu -- prefix index of admitted prompts (host side), the
// counterpart of RadixKVCache (server/radix_kv_cache.h:16-38,
// server/radix_kv_cache.cpp:39-98).
//
// Semantics per token position, as the reference's per-token trie:
//   * insert_prefix(req, tokens): every position on the path gains one
//     reference; positions the path creates record req as their source
//     (cpp:61-81).  The request's token list is remembered (a second insert
//     under the same id replaces the list without releasing the first path,
//     as the reference's map assignment does).
//   * match_prefix(tokens) -> (positions matched from the root, source of the
//     deepest matched position) (cpp:39-59); (0, -1) when nothing matches.
//   * release_prefix(req): one reference less on every position of the
//     remembered path that still exists, then every subtree whose first
//     position has no reference left is removed (cpp:83-98, 20-35).
//
// Layout: a path-compressed radix tree.  An edge holds a run of tokens that
// share one (references, source) pair, so a long prompt is one node instead
// of one node per token; an edge is split where an insert or a release
// covers only its first part, which keeps every position's pair exactly as
// the per-token trie would have it.
#include <cstdint>
#include <memory>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "common.cuh"

struct specdec_radix {
    struct Node {
        std::vector<int32_t> edge;  // tokens from the parent to this node
        int32_t source = -1;
        int64_t refs = 0;
        std::unordered_map<int32_t, std::unique_ptr<Node>> children;  // by first edge token
    };
    Node root;
    std::unordered_map<int32_t, std::vector<int32_t>> history;
    std::mutex mu;
};

namespace specdec {
namespace {
using RNode = specdec_radix::Node;

size_t common_run(const std::vector<int32_t>& edge, const int32_t* t, size_t n) {
    size_t l = 0;
    while (l < edge.size() && l < n && edge[l] == t[l]) ++l;
    return l;
}

// Splits `child` (in parent->children) after its first l tokens; returns the
// node holding those l tokens (same references and source).
RNode* split(RNode* parent, RNode* child, size_t l) {
    auto head = std::make_unique<RNode>();
    head->edge.assign(child->edge.begin(), child->edge.begin() + (long)l);
    head->source = child->source;
    head->refs = child->refs;
    auto& slot = parent->children[child->edge[0]];
    std::unique_ptr<RNode> tail = std::move(slot);
    tail->edge.erase(tail->edge.begin(), tail->edge.begin() + (long)l);
    const int32_t key = tail->edge[0];
    head->children.emplace(key, std::move(tail));
    RNode* h = head.get();
    slot = std::move(head);
    return h;
}

void collect(RNode* node) {
    for (auto it = node->children.begin(); it != node->children.end();) {
        if (it->second->refs == 0) {
            it = node->children.erase(it);
        } else {
            collect(it->second.get());
            ++it;
        }
    }
}

void count(const RNode* node, int64_t* nodes, int64_t* positions) {
    for (const auto& kv : node->children) {
        ++*nodes;
        *positions += (int64_t)kv.second->edge.size();
        count(kv.second.get(), nodes, positions);
    }
}
}  // namespace
}  // namespace specdec

using namespace specdec;

extern "C" int specdec_radix_create(specdec_radix** out) {
    SD_CHECK(out, SPECDEC_EINVAL, "radix_create: null argument");
    *out = new specdec_radix();
    (*out)->root.refs = 1;  // the root is always alive
    return SPECDEC_OK;
}

extern "C" int specdec_radix_destroy(specdec_radix* r) {
    delete r;
    return SPECDEC_OK;
}

extern "C" int specdec_radix_match(specdec_radix* r, const int32_t* tokens, int n, int32_t* matched,
                                   int32_t* source) {
    SD_CHECK(r && (tokens || n == 0) && n >= 0 && matched && source, SPECDEC_EINVAL, "radix_match: bad argument");
    std::lock_guard<std::mutex> lock(r->mu);
    const RNode* node = &r->root;
    size_t i = 0;
    int32_t src = -1;
    while (i < (size_t)n) {
        auto it = node->children.find(tokens[i]);
        if (it == node->children.end()) break;
        const RNode* child = it->second.get();
        const size_t l = common_run(child->edge, tokens + i, (size_t)n - i);
        i += l;
        if (child->source != -1) src = child->source;
        if (l < child->edge.size()) break;
        node = child;
    }
    *matched = (int32_t)i;
    *source = src;
    return SPECDEC_OK;
}

extern "C" int specdec_radix_insert(specdec_radix* r, int32_t request_id, const int32_t* tokens, int n) {
    SD_CHECK(r && (tokens || n == 0) && n >= 0, SPECDEC_EINVAL, "radix_insert: bad argument");
    std::lock_guard<std::mutex> lock(r->mu);
    r->history[request_id].assign(tokens, tokens + n);
    RNode* node = &r->root;
    size_t i = 0;
    while (i < (size_t)n) {
        auto it = node->children.find(tokens[i]);
        if (it == node->children.end()) {
            auto leaf = std::make_unique<RNode>();
            leaf->edge.assign(tokens + i, tokens + n);
            leaf->source = request_id;
            leaf->refs = 1;
            node->children.emplace(tokens[i], std::move(leaf));
            break;
        }
        RNode* child = it->second.get();
        const size_t l = common_run(child->edge, tokens + i, (size_t)n - i);
        if (l < child->edge.size()) child = split(node, child, l);
        child->refs++;
        i += l;
        node = child;
    }
    return SPECDEC_OK;
}

extern "C" int specdec_radix_release(specdec_radix* r, int32_t request_id) {
    SD_CHECK(r, SPECDEC_EINVAL, "radix_release: null argument");
    std::lock_guard<std::mutex> lock(r->mu);
    auto h = r->history.find(request_id);
    if (h == r->history.end()) return SPECDEC_OK;
    const std::vector<int32_t> toks = std::move(h->second);
    r->history.erase(h);
    RNode* node = &r->root;
    size_t i = 0;
    while (i < toks.size()) {
        auto it = node->children.find(toks[i]);
        if (it == node->children.end()) break;
        RNode* child = it->second.get();
        const size_t l = common_run(child->edge, toks.data() + i, toks.size() - i);
        const bool diverged = l < child->edge.size();
        if (diverged) child = split(node, child, l);
        child->refs--;
        if (diverged) break;
        i += l;
        node = child;
    }
    collect(&r->root);
    return SPECDEC_OK;
}

extern "C" int specdec_radix_stats(specdec_radix* r, int64_t* nodes, int64_t* positions) {
    SD_CHECK(r && nodes && positions, SPECDEC_EINVAL, "radix_stats: null argument");
    std::lock_guard<std::mutex> lock(r->mu);
    *nodes = 0;
    *positions = 0;
    count(&r->root, nodes, positions);
    return SPECDEC_OK;
}
