"""Per-token prefix trie restating RadixKVCache (server/radix_kv_cache.cpp:
39-98).

TEST INFRASTRUCTURE ONLY: the checker for the library's path-compressed index
(tests/test_radix.py); pinned against the reference's own class by
tests/golden/radix_golden.npz.  The product path never imports it.
"""
from __future__ import annotations


class _Node:
    __slots__ = ("source", "refs", "children")

    def __init__(self, source=-1, refs=0):
        self.source, self.refs, self.children = source, refs, {}


class RadixTrie:
    def __init__(self):
        self.root = _Node(refs=1)
        self.history = {}

    def match_prefix(self, tokens):
        node, n, src = self.root, 0, -1
        for t in tokens:
            nxt = node.children.get(t)
            if nxt is None:
                break
            node, n = nxt, n + 1
            if node.source != -1:
                src = node.source
        return n, src

    def insert_prefix(self, req, tokens):
        self.history[req] = list(tokens)
        node = self.root
        for t in tokens:
            nxt = node.children.get(t)
            if nxt is None:
                nxt = node.children[t] = _Node(source=req, refs=1)
            else:
                nxt.refs += 1
            node = nxt

    def release_prefix(self, req):
        toks = self.history.pop(req, None)
        if toks is None:
            return
        node = self.root
        for t in toks:
            nxt = node.children.get(t)
            if nxt is None:
                break
            nxt.refs -= 1
            node = nxt

        def gc(n):
            for k in list(n.children):
                c = n.children[k]
                if c.refs == 0:
                    del n.children[k]
                else:
                    gc(c)

        gc(self.root)

    def positions(self):
        def cnt(n):
            return sum(1 + cnt(c) for c in n.children.values())

        return cnt(self.root)
