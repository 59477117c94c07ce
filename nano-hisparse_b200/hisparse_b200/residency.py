"""Indexed residency control for the reference's HybridKVCache.

The reference's residency policy answers three per-(request, layer)
questions by scanning every page or every resident block of the whole
cache (nano_hisparse/hybrid.py):

  * which pages of a layer are resident — resolve pins them before each
    lease (hybrid.py:423-427), a scan over every materialised page;
  * how many pages of a layer are resident — update_residency's hot-demand
    test, per layer (hybrid.py:276-277), again over every page, so one
    policy tick costs O(layers x pages) and each append of a new page runs
    several ticks (hybrid.py:384 and the _slot loop, :335-368);
  * which resident pages of a layer are history that may be unpinned —
    _historical_pages(group) (hybrid.py:204-223), a walk of the allocator's
    whole LRU once per layer per tick.

At configuration 2 (16 requests x 32 layers x 2,048 pages) the first two are
scans of a million Page objects per call. ``install`` keeps, on each
DeviceAllocator, an index from (request, layer) to that layer's resident
page keys in allocator LRU order, maintained where the LRU itself changes
(DeviceAllocator.bind / release, allocator.py:31-53), and replaces the three
scanning methods with versions that read the index: each question then
costs the size of the layer's own resident set. Everything else — the
policy's decisions, its order of unpinning and transitions, the stats, the
events — is the reference's, so a cache behaves identically with or without
the index.

Invariant used: a page has a slot exactly while its key is in the
allocator's LRU (HostStore.bind and HostStore.detach, storage.py:236-255,
are the only writers of Page.slot, and they call allocator.bind /
release). Hot-region blocks are in the LRU under keys with a negative page
index and are never in the index.
"""

from __future__ import annotations

import importlib

_generation = 0  # bumped by every install/uninstall: an older index is stale
_saved: dict = {}


def _state(allocator):
    """(resident, pinned): (request, layer) -> {page key: slot}. `resident`
    holds the layer's resident pages in the allocator's LRU order; `pinned`
    those whose block still holds its allocation reference (not in the
    allocator's reclaimable set). Built from the allocator on first use
    after an install, and rebuilt when the reclaimable set's size is not the
    one the hooks account for (a caller that edits it directly, as one of the
    reference's policy tests does to re-pin a block)."""
    state = allocator.__dict__.get("_hs_group_index")
    if (state is None or state[0] != _generation
            or state[3][0] != len(allocator.reclaimable)):
        resident: dict = {}
        pinned: dict = {}
        for key, slot in allocator.lru.items():
            if key[2] >= 0:
                resident.setdefault(key[:2], {})[key] = slot
                if slot not in allocator.reclaimable:
                    pinned.setdefault(key[:2], {})[key] = slot
        state = (_generation, resident, pinned, [len(allocator.reclaimable)])
        allocator.__dict__["_hs_group_index"] = state
    return state[1], state[2]


def _count_reclaimable(allocator, delta):
    allocator.__dict__["_hs_group_index"][3][0] += delta


def _index(allocator) -> dict:
    return _state(allocator)[0]


def _drop(index, key):
    group = index.get(key[:2])
    if group is not None:
        group.pop(key, None)
        if not group:
            del index[key[:2]]


def _make_bind(original):
    def bind(self, slot, key):
        original(self, slot, key)
        if key[2] >= 0:
            resident, pinned = _state(self)
            resident.setdefault(key[:2], {})[key] = slot
            pinned.setdefault(key[:2], {})[key] = slot  # bound with its allocation reference
    return bind


def _make_release(original):
    def release(self, slot, fence):
        key = self.slots[slot].owner
        resident, pinned = _state(self)
        was = slot in self.reclaimable
        original(self, slot, fence)
        if was:
            _count_reclaimable(self, -1)
        if key is not None and key[2] >= 0:
            _drop(resident, key)
            _drop(pinned, key)
    return release


def _make_unpin(original):
    def unpin(self, slot, on_reuse):
        _, pinned = _state(self)
        was = slot in self.reclaimable
        original(self, slot, on_reuse)
        if not was and slot in self.reclaimable:
            _count_reclaimable(self, 1)
        key = self.slots[slot].owner
        if key is not None and key[2] >= 0:
            _drop(pinned, key)  # now reclaimable
    return unpin


def resident_keys(cache, group):
    """Keys of the resident pages of (request, layer), in LRU order."""
    return _index(cache.allocator).get(group, {})


def historical_pages(self, group=None):
    """hybrid.py:204-223 — sealed, unleased pages at least two behind the
    write tail, in allocator LRU order; for one group, walks only that
    group's resident keys."""
    keys = self.allocator.lru if group is None else list(resident_keys(self, group))
    return _historical_of(self, keys, group)


def _historical_of(self, keys, group):
    """The historical-page filter of hybrid.py:208-222 over `keys`."""
    storage, allocator = self.storage, self.allocator
    found = []
    for key in keys:
        if key[2] < 0 or (group is not None and key[:2] != group):
            continue
        page = storage.pages[key]
        tail = (storage.requests[key[0]].lengths[key[1]] - 1) // self.config.page_size
        if self._writing_key is not None and self._writing_key[:2] == key[:2]:
            tail = self._writing_key[2]
        held = int(page.slot not in allocator.reclaimable)
        if page.sealed and allocator.slots[page.slot].ref_cnt == held \
                and key[2] <= tail - self._hs_tail_pages:
            found.append(page)
    return found


def unpin_clean_pages(self, group):
    """hybrid.py:237-247 — unpin, tail first, the layer's clean historical
    pages that still hold their allocation reference. Only pinned pages can
    be unpinned, so the candidates are taken from the layer's pinned pages
    (the reference takes every historical page and skips the reclaimable
    ones): the same pages in the same order."""
    if not self.tables[group].blocks:
        return
    pinned = _state(self.allocator)[1].get(group)
    if not pinned:
        return
    candidates = _historical_of(self, list(pinned), group)
    reclaimable = self.allocator.reclaimable
    for page in sorted(candidates, key=lambda p: -p.key[2]):
        if (page.host_committed_version == page.content_version
                and page.slot not in reclaimable):
            self.allocator.unpin(page.slot, self._on_block_reused)
            self.storage.stats["clean_page_unpins"] += 1


def update_residency(self, request_id=None, layer=None, *, upcoming_allocation=False):
    """hybrid.py:256-296 with the per-layer resident count read from the
    index: publish finished host mirrors, unpin clean history, raise hot
    demand on the free-block watermark or the resident window, transition
    layers that need their hot region."""
    self.storage.check_stream()
    self._publish_clean()
    groups = [g for g in self.tables
              if g[0] in self.storage.requests
              and (request_id is None or g[0] == request_id)
              and (layer is None or g[1] == layer)]
    for group in groups:
        self._unpin_clean_pages(group)
    for group in groups:
        tables = self.tables[group]
        residents = len(resident_keys(self, group))
        if not residents:
            continue
        if not tables.hot_required:
            free = len(self._available_blocks()) - int(upcoming_allocation)
            if free < self.transition_watermark:
                self._require_hot(group, "watermark")
            elif residents >= self.hot_config.resident_window_pages:
                self._require_hot(group, "window")
        if tables.hot_required and not tables.blocks and not tables.busy:
            try:
                self.transition_to_host(*group)
            except self._hs_capacity_error:
                pass  # retried at the next tick; mappings and demand stay
        self._unpin_clean_pages(group)


def pinned_pages(self, request_id, layer):
    """The pages resolve pins for a lease (hybrid.py:423-427)."""
    pages = self.storage.pages
    return [pages[key] for key in resident_keys(self, (request_id, layer))]


class _PinnedView(dict):
    """storage.pages for the duration of one resolve call: every lookup goes
    to the real mapping; values() yields only the layer's resident pages,
    which are exactly the pages resolve's one scan keeps."""

    __slots__ = ("_real", "_pinned")

    def __init__(self, real, pinned):
        super().__init__()
        self._real, self._pinned = real, pinned

    def values(self):
        return list(self._pinned)

    def __getitem__(self, key):
        return self._real[key]

    def get(self, key, default=None):
        return self._real.get(key, default)

    def __contains__(self, key):
        return key in self._real

    def __len__(self):
        return len(self._real)

    def __iter__(self):
        return iter(self._real)

    def items(self):
        return self._real.items()

    def keys(self):
        return self._real.keys()

    # writes go to the real mapping too (resolve makes none)
    def __setitem__(self, key, value):
        self._real[key] = value

    def __delitem__(self, key):
        del self._real[key]

    def pop(self, key, *default):
        return self._real.pop(key, *default)

    def setdefault(self, key, default=None):
        return self._real.setdefault(key, default)


def _make_resolve(original):
    """resolve (hybrid.py:412-469) with its page scan answered by the index:
    the reference's method runs unchanged against a view of storage.pages
    whose values() are the layer's resident pages. The view is in place only
    for the call, on the calling thread's cache object; like the reference's
    cache, a cache is not to be used from two threads at once."""
    def resolve(self, request_id, layer, topk):
        storage = self.storage
        real = storage.pages
        storage.pages = _PinnedView(real, pinned_pages(self, request_id, layer))
        try:
            return original(self, request_id, layer, topk)
        finally:
            storage.pages = real
    return resolve


def install(package) -> list[str]:
    """Installs the index and the indexed methods into an imported reference
    package; returns the names replaced. Caches created before the call are
    indexed from their allocator's LRU at first use."""
    global _generation
    _generation += 1
    hybrid = importlib.import_module(f"{package.__name__}.hybrid")
    allocator = importlib.import_module(f"{package.__name__}.allocator")
    config = importlib.import_module(f"{package.__name__}.config")
    cache_cls, alloc_cls = hybrid.HybridKVCache, allocator.DeviceAllocator
    replacements = [
        (alloc_cls, "bind", _make_bind),
        (alloc_cls, "release", _make_release),
        (alloc_cls, "unpin", _make_unpin),
        (cache_cls, "_historical_pages", lambda original: historical_pages),
        (cache_cls, "_unpin_clean_pages", lambda original: unpin_clean_pages),
        (cache_cls, "update_residency", lambda original: update_residency),
        (cache_cls, "resolve", _make_resolve),
    ]
    done = []
    for owner, name, make in replacements:
        key = (package.__name__, owner.__name__, name)
        if key not in _saved:
            _saved[key] = (owner, owner.__dict__[name])
        setattr(owner, name, make(_saved[key][1]))
        done.append(f"{owner.__name__}.{name}")
    cache_cls._hs_tail_pages = hybrid.ACTIVE_TAIL_PAGES
    cache_cls._hs_capacity_error = config.CapacityError
    return done


def uninstall(package) -> None:
    """Restores the reference's methods."""
    global _generation
    _generation += 1
    for key, (owner, original) in list(_saved.items()):
        if key[0] == package.__name__:
            setattr(owner, key[2], original)
            del _saved[key]
