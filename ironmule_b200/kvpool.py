"""Paged KV manager with shared prompt prefixes, for the device engine's page tables.

The reference keeps one KV pool for all sequences and lets a new request share the cells of the longest prompt
prefix that any running or finished sequence holds, computing only the rest; finished sequences stay as a cache
and are evicted least recently used first when a request needs room (`SharedPool`,
ironmule/ggml_engine.py:280-432, its prefix trie at :218-278). Here the unit is a page of 16 KV slots, the
granularity the attention kernels read through the page table: a request shares the FULL pages of its longest
cached prefix, links them into its page-table row, and computes only the tokens after them. A position's K/V depend
only on the tokens up to it, so pages are indexed as a trie of pages: an indexed page has a node id (never reused)
and is found under (its parent page's node id, its own 16 tokens), so a lookup or a commit costs O(tokens) and equal
paths mean equal K/V bits. A child indexed under an evicted parent is unreachable, never mistaken for another chain. Shared pages are never written again: every shared slot lies below the request's first
written position (`lead` below). Pages are reference-counted; pages that no running sequence holds stay indexed as
a cache until evicted, deepest page of a chain first.

One pool hands out physical page ids for both models of a speculative pair (each model's cache is indexed the same
way), so it serves the target's and the draft's page tables at once.
"""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field

PAGE = 16


@dataclass
class _Seq:
    pages: list[int] = field(default_factory=list)  # physical pages, in position order
    tokens: list[int] = field(default_factory=list)  # the tokens whose K/V its pages hold, from position 0
    indexed: int = 0  # leading pages entered in (or taken from) the prefix index


class PagePool:
    """`pages` physical pages for `slots` sequence slots, each a page-table row of `row_pages` entries.

    `lead`: how many trailing prompt tokens a request always computes itself (the reference keeps one,
    ggml_engine.py:355; the speculative engine keeps two, since its first draft pass rewrites the K/V of the
    second-to-last committed token)."""

    def __init__(self, pages: int, slots: int, row_pages: int, lead: int = 1):
        if pages < 1 or slots < 1 or row_pages < 1 or lead < 1:
            raise ValueError("pages, slots, row_pages and lead must be positive")
        self.pages, self.slots, self.row_pages, self.lead = pages, slots, row_pages, lead
        self.free: list[int] = list(range(pages - 1, -1, -1))  # popped from the end: page 0 first
        self.ref: dict[int, int] = {}  # page -> running sequences that hold it (absent: free or cached)
        self.index: dict[tuple[int, tuple[int, ...]], int] = {}  # (parent node, the page's tokens) -> page
        self.key_of: dict[int, tuple[int, tuple[int, ...]]] = {}  # indexed page -> its key
        self.node_of: dict[int, int] = {}  # indexed page -> its node id (0 is the root)
        self._next_node = 1
        self.cached: OrderedDict[int, None] = OrderedDict()  # indexed pages nobody holds, evicted first to last
        self.seqs: dict[int, _Seq] = {}
        self.shared_tokens = 0

    # ---- placement ----------------------------------------------------------------------------------------
    def longest(self, ids) -> list[int]:
        """The indexed pages that hold the longest full-page prefix of `ids`, in position order."""
        ids = list(ids)
        out, parent = [], 0
        for j in range(len(ids) // PAGE):
            page = self.index.get((parent, tuple(ids[j * PAGE:(j + 1) * PAGE])))
            if page is None:
                break
            out.append(page)
            parent = self.node_of[page]
        return out

    def _unindex(self, page: int) -> None:
        del self.index[self.key_of.pop(page)]
        del self.node_of[page]

    def _index(self, key, page: int) -> None:
        old = self.key_of.get(page)
        if old is None:
            self.node_of[page] = self._next_node
            self._next_node += 1
        else:  # re-keyed under a live parent (its old parent was evicted); its node id, and so its children, stay
            del self.index[old]
        self.index[key] = page
        self.key_of[page] = key

    def _take(self) -> int:
        if self.free:
            return self.free.pop()
        page, _ = self.cached.popitem(last=False)  # the least recently released, deepest first
        self._unindex(page)
        return page

    def place(self, ids, limit: int, slot: int | None = None) -> tuple[int, int] | None:
        """A slot for a request with prompt `ids` that may grow by `limit` more tokens (its pages are taken now),
        and how many leading prompt tokens its pages already hold; None, with nothing changed, while it does not
        fit (the reference's `SharedPool.place`, ggml_engine.py:352-389). `slot` picks the slot, else the lowest
        free one."""
        ids = list(ids)
        if not ids:
            raise ValueError("an empty prompt")
        if limit < 0:
            raise ValueError("a negative limit")
        total = -(-(len(ids) + limit) // PAGE)
        if total > self.row_pages:
            raise ValueError(f"{len(ids) + limit} tokens exceed a page-table row of {self.row_pages} pages")
        if slot is None:
            free_slots = [s for s in range(self.slots) if s not in self.seqs]
            if not free_slots:
                return None
            slot = free_slots[0]
        elif not 0 <= slot < self.slots or slot in self.seqs:
            raise ValueError(f"slot {slot} is not a free slot")
        shared = self.longest(ids)
        while shared and len(shared) * PAGE > len(ids) - self.lead:
            shared.pop()
        need = total - len(shared)
        revived = sum(1 for p in shared if p not in self.ref)  # cached pages this request takes back
        if len(self.free) + len(self.cached) - revived < need:
            return None
        for p in shared:
            if p in self.ref:
                self.ref[p] += 1
            else:
                del self.cached[p]
                self.ref[p] = 1
        own = []
        for _ in range(need):
            page = self._take()
            self.ref[page] = 1
            own.append(page)
        keep = len(shared) * PAGE
        self.seqs[slot] = _Seq(pages=shared + own, tokens=ids[:keep], indexed=len(shared))
        self.shared_tokens += keep
        return slot, keep

    def row(self, slot: int, width: int | None = None) -> list[int]:
        """The slot's page-table row of `width` entries (row_pages by default): its pages, then its last page
        repeated (those entries lie past every position the sequence may reach and are never read)."""
        pages = self.seqs[slot].pages
        width = self.row_pages if width is None else width
        if width < len(pages):
            raise ValueError("the row is narrower than the slot's pages")
        return pages + [pages[-1]] * (width - len(pages))

    # ---- progress and release -------------------------------------------------------------------------------
    def commit(self, slot: int, tokens) -> None:
        """The slot's pages now hold the final K/V of `tokens` from position 0 (a prefix of what it will hold):
        index its newly completed pages for later requests (the reference's `sync`, ggml_engine.py:391-409,
        without truncation: an indexed page's K/V are final)."""
        tokens = list(tokens)
        seq = self.seqs[slot]
        if len(tokens) > len(seq.pages) * PAGE:
            raise ValueError("more tokens than the slot's pages hold")
        fixed = seq.indexed * PAGE
        if len(tokens) < fixed or tokens[:fixed] != seq.tokens[:fixed]:
            raise ValueError("the tokens contradict the slot's indexed pages")
        seq.tokens = tokens
        parent = 0
        for j in range(len(tokens) // PAGE):  # walk the trie; index this slot's page where the chain has none
            key = (parent, tuple(tokens[j * PAGE:(j + 1) * PAGE]))
            page = self.index.get(key)
            if page is None:
                page = seq.pages[j]
                self._index(key, page)
            parent = self.node_of[page]
        seq.indexed = len(tokens) // PAGE

    def release(self, slot: int, keep: bool = True) -> None:
        """The request in `slot` ends: its indexed pages stay cached (keep) or are dropped from the index, and the
        rest are freed (the reference's `release`, ggml_engine.py:411-427)."""
        seq = self.seqs.pop(slot)
        for page in reversed(seq.pages):  # deepest first, so eviction takes a chain from its end
            count = self.ref[page] - 1
            if count:
                self.ref[page] = count
                continue
            del self.ref[page]
            if page in self.key_of and keep:
                self.cached[page] = None
            else:
                if page in self.key_of:
                    self._unindex(page)
                self.free.append(page)

    def held(self, slot: int) -> bool:
        return slot in self.seqs

    @property
    def used(self) -> int:
        """Pages that running sequences hold."""
        return len(self.ref)

    def summary(self) -> dict:
        return {"pages": self.pages, "used": self.used, "cached": len(self.cached), "free": len(self.free),
                "running": len(self.seqs), "shared_tokens": self.shared_tokens}
