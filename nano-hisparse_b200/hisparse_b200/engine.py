"""Batched decode engine: the reference's scheduler with one batched forward
per step.

``BatchedEngine`` keeps the API and the step semantics of
nano_hisparse/engine.py:24-143 (``add_request`` / ``step`` / ``run`` /
``cancel``; at most one prompt admitted per step; every running request gets
one decode turn per step, in queue order; the same emitted list). What
changes is how a step's decode turns run. The reference calls Model.decode
once per request (model.py:181-221), a chain of small GEMMs and one hot-path
pass per (request, layer). Here all running requests go through each layer
together:

  RMSNorm -> one fused q/k/v GEMM -> RoPE at each request's own position
  -> one hs_append_rows launch (each request's new K/V row into its tail
     block and its host block, with the page's Quest min/max and mean)
  -> DecodeBatch.layer (batched Quest selection, resolver, miss gather,
     two-phase attention)
  -> o_proj GEMM + residual -> RMSNorm -> fused gate/up GEMM -> down GEMM

and one device->host copy of the B argmax tokens ends the step. Prefill
(one prompt per step, as in the reference) runs the dense causal attention
of model.py:165-179 and writes every prompt page in one append launch per
layer.

``ServingCache`` is the cache the engine decodes from: the shared GPU pool
and pinned host store of ``RowCache``, per-request Quest metadata, and the
placement that the reference's HybridKVCache decides on the host
(hybrid.py:161-368) in a simpler form that keeps its guarantees: admission
reserves each layer's hot region and two tail blocks (hybrid.py:43-45), every
page lives in the host store, the two pages at the write tail stay resident,
and older pages stay resident while the pool has unreserved blocks
(borrowed, revoked when an admission needs them). Placement decides only
where rows are read from; the selected rows and their values, and so the
tokens, do not depend on it.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field
from math import ceil

import torch
from torch.nn import functional as F

from .append import append_chunks
from .batched import DecodeBatch
from .cache import LayerTables, RowCache
from .config import ACTIVE_TAIL_PAGES, CacheConfig, CapacityError, HotConfig


@dataclass
class Request:
    """One generation request (engine.py:12-21)."""

    request_id: str
    prompt: list[int]
    max_new_tokens: int
    generated: list[int] = field(default_factory=list)
    prefill_count: int = 0
    decode_count: int = 0
    finished: bool = False
    cancelled: bool = False


@dataclass
class DecoderConfig:
    """Dimensions of the Qwen2-shaped decoder (model.py:18-40), same fields."""

    vocab_size: int = 256
    hidden_size: int = 128
    intermediate_size: int = 256
    num_hidden_layers: int = 2
    num_attention_heads: int = 4
    num_key_value_heads: int = 2
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0

    @property
    def head_dim(self):
        return self.hidden_size // self.num_attention_heads

    def __post_init__(self):
        if (self.hidden_size % self.num_attention_heads
                or self.num_attention_heads % self.num_key_value_heads or self.head_dim % 2):
            raise ValueError("model dimensions must support grouped-query attention and RoPE")


_CONFIG_FIELDS = ("vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
                  "num_attention_heads", "num_key_value_heads", "rms_norm_eps", "rope_theta")


def _layer_keys(i):
    base = f"model.layers.{i}."
    return {
        "input_norm": base + "input_layernorm.weight",
        "post_norm": base + "post_attention_layernorm.weight",
        "q_w": base + "self_attn.q_proj.weight", "q_b": base + "self_attn.q_proj.bias",
        "k_w": base + "self_attn.k_proj.weight", "k_b": base + "self_attn.k_proj.bias",
        "v_w": base + "self_attn.v_proj.weight", "v_b": base + "self_attn.v_proj.bias",
        "o_w": base + "self_attn.o_proj.weight",
        "gate_w": base + "mlp.gate_proj.weight", "up_w": base + "mlp.up_proj.weight",
        "down_w": base + "mlp.down_proj.weight",
    }


class DecoderWeights:
    """The decoder's parameters as plain tensors, under the state_dict names
    of the reference model (model.py:43-97), which are also those of a
    Hugging Face Qwen2 checkpoint. q/k/v and gate/up are kept fused for the
    batched GEMMs."""

    def __init__(self, config: DecoderConfig, state: dict, device=None, dtype=None):
        self.config = config
        first = state["model.embed_tokens.weight"]
        self.device = torch.device(device) if device is not None else first.device
        self.dtype = dtype if dtype is not None else first.dtype

        def get(name):
            return state[name].to(device=self.device, dtype=self.dtype).contiguous()

        self.embed = get("model.embed_tokens.weight")
        self.norm = get("model.norm.weight")
        self.lm_head = get("lm_head.weight")
        self.layers = []
        for i in range(config.num_hidden_layers):
            key = _layer_keys(i)
            w = {name: get(k) for name, k in key.items()}
            self.layers.append({
                "input_norm": w["input_norm"], "post_norm": w["post_norm"],
                "qkv_w": torch.cat((w["q_w"], w["k_w"], w["v_w"])).contiguous(),
                "qkv_b": torch.cat((w["q_b"], w["k_b"], w["v_b"])).contiguous(),
                "o_w": w["o_w"],
                "gate_up_w": torch.cat((w["gate_w"], w["up_w"])).contiguous(),
                "down_w": w["down_w"],
            })
        cfg = config
        self.inv_freq = cfg.rope_theta ** (
            -torch.arange(0, cfg.head_dim, 2, device=self.device).float() / cfg.head_dim)

    @classmethod
    def from_model(cls, model, device=None, dtype=None):
        """From a reference ``Model`` (or any module with its state_dict names
        and a config carrying the DecoderConfig fields)."""
        cfg = DecoderConfig(**{name: getattr(model.config, name) for name in _CONFIG_FIELDS})
        return cls(cfg, model.state_dict(), device, dtype)

    @classmethod
    def random(cls, config: DecoderConfig, seed: int, device="cuda", dtype=torch.bfloat16):
        """Seeded weights that come out identical on every machine: integers
        from torch's CPU generator scaled by powers of two, so every value is
        exact in fp32 (linear weights uniform in +-1/sqrt(fan_in) rounded to
        1/4096 steps, biases and norm offsets smaller)."""
        g = torch.Generator().manual_seed(seed)
        cfg = config

        def uniform(shape, scale):
            ints = torch.randint(-4096, 4097, shape, generator=g, dtype=torch.int64)
            return ints.to(torch.float32) * (scale / 4096.0)

        def pow2_scale(fan_in):  # the power of two nearest 1/sqrt(fan_in)
            return 2.0 ** round(-0.5 * torch.log2(torch.tensor(float(fan_in))).item())

        h, kvw = cfg.hidden_size, cfg.num_key_value_heads * cfg.head_dim
        state = {"model.embed_tokens.weight": uniform((cfg.vocab_size, h), 1.0)}
        for i in range(cfg.num_hidden_layers):
            key = _layer_keys(i)
            state[key["input_norm"]] = 1.0 + uniform((h,), 1 / 8)
            state[key["post_norm"]] = 1.0 + uniform((h,), 1 / 8)
            for name, rows in (("q", h), ("k", kvw), ("v", kvw)):
                state[key[name + "_w"]] = uniform((rows, h), pow2_scale(h))
                state[key[name + "_b"]] = uniform((rows,), 1 / 16)
            state[key["o_w"]] = uniform((h, h), pow2_scale(h))
            state[key["gate_w"]] = uniform((cfg.intermediate_size, h), pow2_scale(h))
            state[key["up_w"]] = uniform((cfg.intermediate_size, h), pow2_scale(h))
            state[key["down_w"]] = uniform((h, cfg.intermediate_size),
                                           pow2_scale(cfg.intermediate_size))
        state["model.norm.weight"] = 1.0 + uniform((h,), 1 / 8)
        state["lm_head.weight"] = uniform((cfg.vocab_size, h), pow2_scale(h))
        return cls(cfg, state, device, dtype)

    def state_dict(self):
        """The reference model's state_dict (fp32 copies on the CPU), e.g. to
        load the same weights into a reference ``Model``."""
        cfg, kvw = self.config, self.config.num_key_value_heads * self.config.head_dim
        h = cfg.hidden_size
        out = {"model.embed_tokens.weight": self.embed, "model.norm.weight": self.norm,
               "lm_head.weight": self.lm_head}
        for i, w in enumerate(self.layers):
            key = _layer_keys(i)
            q_w, k_w, v_w = w["qkv_w"].split((h, kvw, kvw))
            q_b, k_b, v_b = w["qkv_b"].split((h, kvw, kvw))
            gate, up = w["gate_up_w"].split((cfg.intermediate_size, cfg.intermediate_size))
            out.update({key["input_norm"]: w["input_norm"], key["post_norm"]: w["post_norm"],
                        key["q_w"]: q_w, key["k_w"]: k_w, key["v_w"]: v_w, key["q_b"]: q_b,
                        key["k_b"]: k_b, key["v_b"]: v_b, key["o_w"]: w["o_w"],
                        key["gate_w"]: gate, key["up_w"]: up, key["down_w"]: w["down_w"]})
        return {k: v.detach().float().cpu().contiguous() for k, v in out.items()}

    # -- the dense math of model.py:45-179, batched over rows ------------------------
    def rms_norm(self, x, weight):
        """model.py:46-55: fp32 normalisation, back to the model dtype, times weight."""
        xf = x.float()
        normalized = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + self.config.rms_norm_eps)
        return normalized.to(x.dtype) * weight

    def project(self, layer, x, positions):
        """model.py:136-155 for rows x [N, hidden] at float positions [N]:
        returns q [N, Hq, D], k and v [N, Hkv, D], RoPE applied to q and k."""
        cfg, w = self.config, self.layers[layer]
        n, d = x.shape[0], cfg.head_dim
        h = self.rms_norm(x, w["input_norm"])
        qkv = F.linear(h, w["qkv_w"], w["qkv_b"])
        hq, hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        q, k, v = qkv.split((hq * d, hkv * d, hkv * d), dim=-1)
        q, k, v = q.view(n, hq, d), k.view(n, hkv, d), v.reshape(n, hkv, d)
        angles = positions[:, None] * self.inv_freq[None, :]
        angles = torch.cat((angles, angles), -1)[:, None, :]
        cosine, sine = angles.cos().to(x.dtype), angles.sin().to(x.dtype)

        def rotate(t):
            a, b = t.chunk(2, -1)
            return t * cosine + torch.cat((-b, a), -1) * sine

        return rotate(q), rotate(k), v

    def finish(self, layer, residual, attention):
        """model.py:157-160: o_proj + residual, then the MLP block."""
        w = self.layers[layer]
        x = residual + F.linear(attention.reshape(residual.shape[0], -1), w["o_w"])
        gate, up = F.linear(self.rms_norm(x, w["post_norm"]), w["gate_up_w"]).chunk(2, -1)
        return x + F.linear(F.silu(gate) * up, w["down_w"])

    def logits(self, x):
        """model.py:179 / 221: fp32 logits of rows x [N, hidden]."""
        return F.linear(self.rms_norm(x, self.norm), self.lm_head).float()


def _staged(values: torch.Tensor, device) -> torch.Tensor:
    """One host->device copy through pinned memory on the current stream (the
    caching host allocator keeps the staging block alive until it completes)."""
    return values.pin_memory().to(device, non_blocking=True)


class _Reservation:
    """One request's share of a ServingCache."""

    def __init__(self, request_id, max_tokens, layers, pages):
        self.request_id, self.max_tokens, self.layers, self.pages = (
            request_id, max_tokens, layers, pages)
        self.length = 0
        self.host = None        # int64 numpy [layers, pages]: host block of each page
        self.hot = None         # int numpy [layers, hot_blocks]
        self.tail = None        # int numpy [layers, 2]: the two tail blocks
        self.tail_page = None   # int numpy [layers, 2]: the page each tail block holds
        self.borrowed = []      # [(layer, page, block)] in borrow order
        self.tables = None      # (source, resident, hot, tags, lru) device tensors
        self.minimum = self.maximum = self.summary = None


class ServingCache:
    """Pool, host store, per-request metadata and placement for BatchedEngine.

    Admission (``reserve``) takes, per layer, the hot region's blocks and
    ACTIVE_TAIL_PAGES tail blocks from the pool (the credits of
    hybrid.py:43-45 and :161-182) and a host block for every page the request
    can reach. Page p is written into tail block p % 2; when page p starts,
    page p - 2 leaves the tail and keeps its block as borrowed history if the
    pool has an unreserved block for the tail, else it becomes host-only.
    Prompt pages before the tail borrow blocks the same way. ``reserve``
    revokes borrowed blocks (oldest first) when the pool is short of credits.
    Every page is also in the host store, so revoking only redirects reads
    to the miss gather. All device-table updates are stream-ordered on the
    compute stream with the kernels that read them."""

    def __init__(self, config: CacheConfig, hot: HotConfig):
        self.config, self.hot_config = config, hot
        self.rows = RowCache(config, hot)
        self.pool, self.host, self.device = self.rows.pool, self.rows.host, self.rows.device
        self.compute, self.transfer = self.rows.compute, self.rows.transfer
        self.hot_blocks = self.rows.hot_blocks
        self.free_pool = list(range(config.gpu_pages))[::-1]  # pop() takes the lowest
        self.free_host = list(range(config.host_pages))[::-1]
        self.requests: dict[str, _Reservation] = {}
        elt = torch.empty((), dtype=config.dtype).element_size()
        self._meta_row = config.kv_heads * config.head_dim
        self._meta_bytes = self._meta_row * elt
        self.stats = {"borrowed": 0, "revoked": 0, "host_only_pages": 0}

    # -- capacity (engine.py:48-62, hybrid.py:125-134) --------------------------------
    @property
    def budget(self):
        return self.config.gpu_pages

    def admission_blocks(self, layers):
        return self.hot_config.admission_blocks(self.config.page_size, layers)

    def index_reservation_bytes(self, max_tokens, layers):
        """Device index bytes of one request: per page source/resident entries
        and Quest min/max and mean metadata, per layer the hot tables."""
        cfg, pages = self.config, ceil(max_tokens / self.config.page_size)
        per_page = 8 + 2 * self._meta_bytes + 4 * self._meta_row
        return layers * (pages * per_page + self.hot_blocks * 4 + self.hot_config.hot_rows * 12)

    @property
    def index_bytes(self):
        return sum(self.index_reservation_bytes(r.max_tokens, r.layers)
                   for r in self.requests.values())

    def _promised(self):
        return sum(self.admission_blocks(r.layers) for r in self.requests.values())

    def reserve(self, request_id, max_tokens, layers):
        """Admit a request (hybrid.py:161-182): CapacityError if its credits,
        host pages or index bytes do not fit now."""
        cfg = self.config
        if request_id in self.requests:
            raise ValueError(f"request {request_id!r} is already reserved")
        pages = ceil(max_tokens / cfg.page_size)
        credits = self.admission_blocks(layers)
        if self._promised() + credits > self.budget:
            raise CapacityError("hot-region + active-tail credits exhausted; defer admission")
        if pages * layers > len(self.free_host):
            raise CapacityError("host pool exhausted; defer admission")
        if self.index_bytes + self.index_reservation_bytes(max_tokens, layers) > \
                cfg.index_budget_bytes:
            raise CapacityError("index budget exhausted; defer admission")
        updates = self._revoke(credits - len(self.free_pool))
        res = _Reservation(request_id, max_tokens, layers, pages)
        res.host = torch.tensor([self.free_host.pop() for _ in range(pages * layers)],
                                dtype=torch.int64).view(layers, pages).numpy()
        res.hot = torch.tensor([self.free_pool.pop() for _ in range(layers * self.hot_blocks)],
                               dtype=torch.int64).view(layers, self.hot_blocks).numpy()
        res.tail = torch.tensor([self.free_pool.pop() for _ in range(layers * ACTIVE_TAIL_PAGES)],
                                dtype=torch.int64).view(layers, ACTIVE_TAIL_PAGES).numpy()
        res.tail_page = res.tail * 0 - 1
        dev, h = self.device, self.hot_config.hot_rows
        with torch.cuda.stream(self.compute):
            self._apply(updates)
            source = _staged(torch.from_numpy(res.host).to(torch.int32), dev)
            resident = torch.full((layers, pages), -1, dtype=torch.int32, device=dev)
            hot = _staged(torch.from_numpy(res.hot).to(torch.int32), dev)
            tags = torch.full((layers, h), -1, dtype=torch.int32, device=dev)
            lru = torch.arange(h, dtype=torch.int64, device=dev).repeat(layers, 1)
            shape = (layers, pages, cfg.kv_heads, cfg.head_dim)
            res.minimum = torch.full(shape, float("inf"), dtype=cfg.dtype, device=dev)
            res.maximum = torch.full(shape, float("-inf"), dtype=cfg.dtype, device=dev)
            res.summary = torch.zeros(shape, dtype=torch.float32, device=dev)
        res.tables = (source, resident, hot, tags, lru)
        for layer in range(layers):
            self.rows.tables[request_id, layer] = LayerTables(
                source[layer], resident[layer], hot[layer], tags[layer], lru[layer],
                blocks=[int(b) for b in res.hot[layer]])
            self.rows.lengths[request_id, layer] = 0
        self.requests[request_id] = res
        return res

    def _revoke(self, need):
        """Take borrowed blocks back (requests in admission order, each one's
        oldest first) until `need` are free; returns the resident-table
        updates."""
        updates = []
        if need <= 0:
            return updates
        if sum(len(res.borrowed) for res in self.requests.values()) < need:
            raise CapacityError("pool blocks exhausted; defer admission")
        for res in self.requests.values():
            while res.borrowed and need > 0:
                layer, page, block = res.borrowed.pop(0)
                updates.append((res, layer, page, -1))
                self.free_pool.append(block)
                self.stats["revoked"] += 1
                need -= 1
        return updates

    def _apply(self, updates):
        """Resident-table writes [(reservation, layer, page, block)] on the
        current stream: one copy and one scatter per request touched."""
        by_request = {}
        for res, layer, page, block in updates:
            by_request.setdefault(id(res), (res, []))[1].append((layer, page, block))
        for res, entries in by_request.values():
            packed = torch.tensor(entries, dtype=torch.int64).t().contiguous()
            staged = _staged(packed, self.device)
            res.tables[1].index_put_((staged[0], staged[1]), staged[2].to(torch.int32))

    def _borrow(self):
        """An unreserved pool block, or None (credits of admitted requests
        were taken at admission, so every free block is unreserved)."""
        return self.free_pool.pop() if self.free_pool else None

    # -- placement and the append metadata of a prompt or a decode step ---------------
    def _pointers(self, res, layer, pages):
        """Device addresses of the min/max/summary entries of `pages` (numpy)."""
        index = layer * res.pages + pages
        return (res.minimum.data_ptr() + index * self._meta_bytes,
                res.maximum.data_ptr() + index * self._meta_bytes,
                res.summary.data_ptr() + index * self._meta_row * 4)

    def _enter_tail(self, res, layer, page, updates):
        """Page `page` starts in tail block page % 2; the page that block held
        keeps it as borrowed history if the pool can replace it, else it
        becomes host-only."""
        slot = page % ACTIVE_TAIL_PAGES
        old = int(res.tail_page[layer, slot])
        if old >= 0 and old != page:
            block = self._borrow()
            if block is not None:
                res.borrowed.append((layer, old, int(res.tail[layer, slot])))
                res.tail[layer, slot] = block
                self.stats["borrowed"] += 1
            else:
                updates.append((res, layer, old, -1))
        res.tail_page[layer, slot] = page
        updates.append((res, layer, page, int(res.tail[layer, slot])))
        return int(res.tail[layer, slot])

    def plan_prompt(self, request_id, tokens):
        """Places a prompt's pages and stages its append metadata: returns
        per-layer device views (within, count, pool_block, host_block,
        minimum/maximum/summary pointers) for one append launch per layer."""
        import numpy as np

        res, cfg = self.requests[request_id], self.config
        if res.length:
            raise ValueError("prefill is allowed exactly once per request")
        if tokens > res.max_tokens:
            raise CapacityError("request exceeds its reserved host capacity")
        P, L = cfg.page_size, res.layers
        n = ceil(tokens / P)
        tail = set(range(max(0, n - ACTIVE_TAIL_PAGES), n))
        blocks = np.full((L, n), -1, dtype=np.int64)
        updates = []
        for page in range(n - 1, -1, -1):  # the most recent history borrows first
            for layer in range(L):
                if page in tail:
                    blocks[layer, page] = self._enter_tail(res, layer, page, updates)
                    continue
                block = self._borrow()
                if block is None:
                    self.stats["host_only_pages"] += 1
                    continue
                res.borrowed.append((layer, page, block))
                self.stats["borrowed"] += 1
                blocks[layer, page] = block
                updates.append((res, layer, page, block))
        pages = np.arange(n)
        words = np.empty(5 * L * n + n, dtype=np.int64)
        meta = words[:5 * L * n].reshape(5, L, n)
        meta[0] = blocks
        meta[1] = res.host[:, :n]
        for layer in range(L):
            meta[2, layer], meta[3, layer], meta[4, layer] = self._pointers(res, layer, pages)
        halves = words[5 * L * n:].view(np.int32)
        halves[:n] = 0
        halves[n:] = np.minimum(P, tokens - pages * P)
        with torch.cuda.stream(self.compute):
            self._apply(updates)
            staged = _staged(torch.from_numpy(words), self.device)
        meta_d = staged[:5 * L * n].view(5, L, n)
        ints = staged[5 * L * n:].view(torch.int32)
        return ints[:n], ints[n:], meta_d

    def plan_decode(self, request_ids, tokens):
        """Places the page each request's next token starts (if any) and
        stages one decode step's inputs in one copy: the token ids, and per
        layer the append metadata of one row per request. Returns (tokens
        int64 [B], within int32 [B], count int32 [B], lengths int32 [B] after
        the append, meta int64 [5, L, B])."""
        import numpy as np

        cfg, P = self.config, self.config.page_size
        reservations = [self.requests[r] for r in request_ids]
        B, L = len(reservations), reservations[0].layers
        words = np.empty(5 * L * B + B + (3 * B + 1) // 2, dtype=np.int64)
        meta = words[:5 * L * B].reshape(5, L, B)
        words[5 * L * B:5 * L * B + B] = tokens
        halves = words[5 * L * B + B:].view(np.int32)
        updates = []
        for b, res in enumerate(reservations):
            position = res.length
            if position >= res.max_tokens:
                raise CapacityError("request exceeds its reserved host capacity")
            page, within = divmod(position, P)
            for layer in range(L):
                if within == 0:
                    self._enter_tail(res, layer, page, updates)
                meta[0, layer, b] = res.tail[layer, page % ACTIVE_TAIL_PAGES]
                meta[1, layer, b] = res.host[layer, page]
                meta[2, layer, b], meta[3, layer, b], meta[4, layer, b] = self._pointers(
                    res, layer, page)
            halves[b] = within
            halves[B + b] = 1
            halves[2 * B + b] = position + 1
        with torch.cuda.stream(self.compute):
            self._apply(updates)
            staged = _staged(torch.from_numpy(words), self.device)
        ints = staged[5 * L * B + B:].view(torch.int32)
        return (staged[5 * L * B:5 * L * B + B], ints[:B], ints[B:2 * B], ints[2 * B:3 * B],
                staged[:5 * L * B].view(5, L, B))

    def append(self, layer, k, v, within, count, meta, mapped=True):
        """One append launch for `layer`: chunk b of k/v [B, T, Hkv, D] goes
        where plan_prompt / plan_decode staged it."""
        append_chunks(k, v, within, count, meta[0, layer], self.pool, meta[2, layer],
                      meta[3, layer], meta[4, layer], self.config,
                      self.rows.mapped if mapped else None, meta[1, layer])

    def advance(self, request_id, tokens):
        """Records `tokens` more rows of history on every layer of a request."""
        res = self.requests[request_id]
        res.length += tokens
        for layer in range(res.layers):
            self.rows.lengths[request_id, layer] = res.length

    def length(self, request_id):
        return self.requests[request_id].length

    # -- release and introspection ----------------------------------------------------
    def release_request(self, request_id, wait=False):
        """Returns a request's blocks (hybrid.py:471-490). Later work that
        reuses them is ordered after this request's reads by the compute
        stream, and gathers wait for the compute stream's resolver."""
        res = self.requests.pop(request_id)
        self.free_host.extend(int(b) for b in res.host.reshape(-1)[::-1])
        blocks = [int(b) for b in res.hot.reshape(-1)] + [int(b) for b in res.tail.reshape(-1)]
        blocks += [block for _, _, block in res.borrowed]
        self.free_pool.extend(sorted(blocks, reverse=True))
        for layer in range(res.layers):
            del self.rows.tables[request_id, layer]
            del self.rows.lengths[request_id, layer]
        if wait:
            self.rows.synchronize()

    def reset_stats(self):
        self.rows.reset_stats()

    def snapshot(self):
        out = self.rows.snapshot()
        out["placement"] = dict(self.stats)
        out["free_pool_blocks"] = len(self.free_pool)
        out["free_host_blocks"] = len(self.free_host)
        return out

    def assert_invariants(self):
        """Block ownership is a partition, and every device resident table
        matches the host's placement (reads the device: tests only)."""
        cfg = self.config
        owned = list(self.free_pool)
        hosts = list(self.free_host)
        for res in self.requests.values():
            owned += [int(b) for b in res.hot.reshape(-1)] + [int(b) for b in res.tail.reshape(-1)]
            owned += [block for _, _, block in res.borrowed]
            hosts += [int(b) for b in res.host.reshape(-1)]
            expected = torch.full((res.layers, res.pages), -1, dtype=torch.int32)
            for layer, page, block in res.borrowed:
                expected[layer, page] = block
            for layer in range(res.layers):
                for slot in range(ACTIVE_TAIL_PAGES):
                    if res.tail_page[layer, slot] >= 0:
                        expected[layer, res.tail_page[layer, slot]] = int(res.tail[layer, slot])
            self.rows.synchronize()
            assert torch.equal(res.tables[1].cpu(), expected), res.request_id
        assert sorted(owned) == list(range(cfg.gpu_pages)), "pool blocks are not a partition"
        assert sorted(hosts) == list(range(cfg.host_pages)), "host blocks are not a partition"


class BatchedEngine:
    """The reference Engine's scheduler (engine.py:24-143) over one batched
    forward per step.

    model: DecoderWeights, or a reference ``Model`` (its weights are read
    once); cache: ServingCache. top_k: Quest page budget per layer (the
    reference's quest_selection top_pages, sink and tail pages included), or
    None for the full causal history. backend is accepted for signature
    parity; every path runs libhisparse. selector: "quest" only (the mean
    indexer of selection.py:127 is not part of this path)."""

    def __init__(self, model, cache: ServingCache, top_k=None, backend="auto",
                 eos_token_id: int | None = None, selector: str = "quest"):
        weights = model if isinstance(model, DecoderWeights) else DecoderWeights.from_model(model)
        cfg, kv = weights.config, cache.config
        if (cfg.num_key_value_heads, cfg.head_dim) != (kv.kv_heads, kv.head_dim):
            raise ValueError("model/cache head dimensions differ")
        if weights.device != cache.pool.device or weights.dtype != cache.pool.dtype:
            raise ValueError("model/cache dtype or device differ")
        if top_k is not None and top_k < 1:
            raise ValueError("top_k must be positive or None")
        if selector != "quest":
            raise ValueError("selector must be quest")
        self.model, self.cache, self.top_k, self.backend = weights, cache, top_k, backend
        self.eos_token_id, self.selector = eos_token_id, selector
        self.requests: dict[str, Request] = {}
        self.waiting: deque[Request] = deque()
        self.running: deque[Request] = deque()
        page = kv.page_size
        self._top_pages = top_k if top_k is not None else \
            cache.hot_config.max_union_rows // page
        if self._top_pages < 1 or self._top_pages * page > cache.hot_config.max_union_rows:
            raise ValueError("top_k * page_size exceeds the cache's max_union_rows")
        self._batch, self._batch_ids, self._lengths = None, None, None
        self._all_positions = None

    # -- engine.py:48-68 ----------------------------------------------------------------
    def add_request(self, request_id, prompt, max_new_tokens=16):
        cfg, cache = self.model.config, self.cache
        if request_id in self.requests or not prompt or max_new_tokens < 1:
            raise ValueError("need a unique ID, nonempty prompt, and positive output length")
        if any(token < 0 or token >= cfg.vocab_size for token in prompt):
            raise ValueError("token outside model vocabulary")
        total = len(prompt) + max_new_tokens
        needed = -(-total // cache.config.page_size)
        if needed * cfg.num_hidden_layers > cache.config.host_pages:
            raise CapacityError("request cannot fit even in an empty host pool")
        if cache.admission_blocks(cfg.num_hidden_layers) > cache.budget:
            raise CapacityError("request hot-region + tail footprint cannot fit the device pool")
        if cache.index_reservation_bytes(total, cfg.num_hidden_layers) > \
                cache.config.index_budget_bytes:
            raise CapacityError("request index cannot fit even in an empty index budget")
        if self.top_k is None and total > self._top_pages * cache.config.page_size:
            raise CapacityError("full-history attention needs the whole request within "
                                "max_union_rows")
        request = Request(request_id, list(prompt), max_new_tokens)
        self.requests[request_id] = request
        self.waiting.append(request)
        return request

    def _emit(self, request, token):
        request.generated.append(token)
        if token == self.eos_token_id or len(request.generated) >= request.max_new_tokens:
            request.finished = True
            self.cache.release_request(request.request_id, wait=False)
        return token

    def step(self):
        """Admit at most one prompt, then give every running request one decode
        turn, all of them in one batched forward (engine.py:76-126). Returns
        [(request_id, token)] in the reference's order."""
        emitted = []
        cfg = self.model.config
        if self.waiting:
            request = self.waiting[0]
            try:
                self.cache.reserve(request.request_id,
                                   len(request.prompt) + request.max_new_tokens,
                                   cfg.num_hidden_layers)
                admitted = True
            except CapacityError:
                if not self.running:  # nothing running will ever free blocks
                    raise
                admitted = False
            if admitted:
                self.waiting.popleft()
                token = self._prefill(request)
                request.prefill_count += 1
                emitted.append((request.request_id, self._emit(request, token)))
                if not request.finished:
                    self.running.append(request)
        batch = list(self.running)
        if batch:
            tokens = self._decode(batch)
            for request, token in zip(batch, tokens):
                request.decode_count += 1
                emitted.append((request.request_id, self._emit(request, token)))
            self.running = deque(r for r in batch if not r.finished)
        return emitted

    def run(self):
        while self.waiting or self.running:
            self.step()
        self.cache.rows.synchronize()
        return {name: request.generated for name, request in self.requests.items()}

    def cancel(self, request_id):
        request = self.requests[request_id]
        if request.finished:
            return
        if request in self.waiting:
            self.waiting.remove(request)
        else:
            self.running.remove(request)
            self.cache.release_request(request_id, wait=False)
        request.finished = request.cancelled = True

    # -- the forward passes ---------------------------------------------------------
    @torch.inference_mode()
    def _prefill(self, request) -> int:
        """model.py:162-179 for one prompt; its K/V pages go to the cache in
        one append launch per layer."""
        w, cache, cfg = self.model, self.cache, self.model.config
        n, P = len(request.prompt), cache.config.page_size
        pages = ceil(n / P)
        groups = cfg.num_attention_heads // cfg.num_key_value_heads
        with torch.cuda.stream(cache.compute):
            within, count, meta = cache.plan_prompt(request.request_id, n)
            x = F.embedding(torch.tensor(request.prompt, device=w.device), w.embed)
            positions = torch.arange(n, device=w.device).float()
            pad = pages * P - n
            for layer in range(cfg.num_hidden_layers):
                q, k, v = w.project(layer, x, positions)
                kp = F.pad(k, (0, 0, 0, 0, 0, pad)).view(pages, P, *k.shape[1:])
                vp = F.pad(v, (0, 0, 0, 0, 0, pad)).view(pages, P, *v.shape[1:])
                cache.append(layer, kp, vp, within, count, meta)
                attention = F.scaled_dot_product_attention(
                    q.transpose(0, 1), k.repeat_interleave(groups, 1).transpose(0, 1),
                    v.repeat_interleave(groups, 1).transpose(0, 1), is_causal=True,
                ).transpose(0, 1)
                x = w.finish(layer, x, attention)
            token = int(w.logits(x[-1:])[0].argmax().item())
        cache.advance(request.request_id, n)
        return token

    def _decode_batch(self, ids):
        """The DecodeBatch of the running set, rebuilt when the set changes."""
        if ids == self._batch_ids:
            return self._batch
        cache, cfg = self.cache, self.model.config
        res = [cache.requests[r] for r in ids]
        with torch.cuda.stream(cache.compute):
            batch = DecodeBatch(cache.rows, ids, cfg.num_hidden_layers,
                                {r.request_id: r.minimum for r in res},
                                {r.request_id: r.maximum for r in res}, self._top_pages,
                                cfg.num_attention_heads, keep_sink=True)
            self._lengths = torch.zeros(len(ids), dtype=torch.int32, device=cache.device)
            batch.bind_lengths(self._lengths)
        self._batch, self._batch_ids = batch, list(ids)
        return batch

    @torch.inference_mode()
    def _decode(self, requests) -> list[int]:
        """One decode turn of every running request: model.py:181-221 batched."""
        w, cache, cfg = self.model, self.cache, self.model.config
        ids = [r.request_id for r in requests]
        batch = self._decode_batch(ids)
        b = len(ids)
        with torch.cuda.stream(cache.compute):
            tokens, within, count, lengths, meta = cache.plan_decode(
                ids, [r.generated[-1] for r in requests])
            self._lengths.copy_(lengths)
            x = F.embedding(tokens, w.embed)
            positions = (lengths - 1).float()
            selected = None
            if self.top_k is None:  # the full causal history (selection.py:127-135)
                width = batch.width
                ar = torch.arange(width, dtype=torch.int32, device=cache.device)
                selected = torch.where(ar[None, :] < lengths[:, None], ar[None, :],
                                       torch.full_like(ar[None, :], -1)).contiguous()
            for layer in range(cfg.num_hidden_layers):
                q, k, v = w.project(layer, x, positions)
                cache.append(layer, k.unsqueeze(1), v.unsqueeze(1), within, count, meta)
                attention = batch.layer(layer, q.contiguous(), positions=selected)
                x = w.finish(layer, x, attention)
            cache.rows.row_stats.add_(batch.last_counts().sum((0, 1)))
            out = w.logits(x).argmax(-1).cpu()
        for r in ids:
            cache.advance(r, 1)
        return out.tolist()
