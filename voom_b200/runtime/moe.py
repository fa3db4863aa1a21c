"""MoE expert SwiGLU on compressed expert pages (fused rANS decode + GEMV).

Expert projections stay in HBM as VRN1 frames (bf16_rans format) with a
checkpoint index; every forward decodes them inside the GEMV kernels.

  ExpertStore      - per-expert gate/up/down pages + the device page table.
  MoeLayer         - one layer on the device: RMSNorm, router, top-k,
                     fused experts, ordered combine, residual
                     (runtime/layer_runner.py:347-394 run_moe_mlp).
  swiglu_grouped   - experts chosen on the host (consume_expert_batches path,
                     runtime/expert_batching.py:13-41).

Reference interface replaced: runtime/layer_runner.py:185-190, 347-394;
runtime/qwen35.py:584-638 (route + consume); runtime/quant.py:431-444.
"""

from __future__ import annotations

import ctypes
import threading

import numpy as np
import torch

from .. import _device
from .._lib import check, load
from ..formats import bf16_rans

PROJ_DTYPE = np.dtype([("src", "<u8"), ("tiles", "<u8"), ("ckpt", "<u8"), ("ckpt_base", "<u8"),
                       ("n_tiles", "<u4"), ("every", "<u4"), ("rows", "<u4"), ("cols", "<u4")])
PAGES_DTYPE = np.dtype([("gate", PROJ_DTYPE), ("up", PROJ_DTYPE), ("down", PROJ_DTYPE)])
assert PAGES_DTYPE.itemsize == 144


MAX_TILES = 65  # tiles per projection the fused kernels take (kSeams + 1 in csrc/moe_proj.cuh)

# Status word bits written by the fused kernels (one u32 per layer).
STATUS_PAGE = 1    # a compressed expert page failed its checkpoint verification
STATUS_ROUTES = 2  # an expert got more route rows than the launch covered
STATUS_GEOMETRY = 4  # page geometry the kernels do not take (segment length, tile size or count)
STATUS_TIMEOUT = 8  # a tensor-core completion wait ran out (reported, never observed)
STATUS_NO_HOLDER = 16  # expert parallelism: a routed expert that no rank holds


def raise_on_status(status: torch.Tensor, what: str) -> None:
    """Reads a layer's device status word (synchronises its stream), clears it,
    and raises ValueError when a kernel reported a fault.  The reference
    raises while decoding a damaged page (formats/bf16_rans.py:216-221); the
    fused kernels cannot raise, so the fault is carried to the next check."""
    v = int(status.item())
    if v:
        status.zero_()
        parts = []
        if v & STATUS_PAGE:
            parts.append("a compressed expert page failed its checkpoint verification")
        if v & STATUS_ROUTES:
            parts.append("an expert had more routed tokens than the launch covered")
        if v & STATUS_GEOMETRY:
            parts.append("an expert page has a geometry the fused kernels do not take")
        if v & STATUS_TIMEOUT:
            parts.append("a tensor-core completion wait ran out")
        if v & STATUS_NO_HOLDER:
            parts.append("a routed expert is held by no rank")
        raise ValueError(f"{what}: " + "; ".join(parts or [f"status 0x{v:x}"]))


EVERY_LARGE = 4 << 20  # projections of this many weights or more take 512-symbol segments


def every_for(rows: int, cols: int, longest: int | None = None) -> int:
    """Checkpoint interval of a rows x cols projection: the longest power of
    two <= `longest` (and >= 64) dividing the row, so a lane pair of the fused
    kernels decodes whole row segments; `longest` is 512 for projections of
    EVERY_LARGE weights or more (they have work items enough, and longer
    segments halve the per-segment setup), else 256 (shorter chains are where a
    small projection's parallelism comes from).  The fused kernels size their
    row blocks from this rule (every_rule in csrc/moe_proj.cuh)."""
    e = longest if longest is not None else (512 if rows * cols >= EVERY_LARGE else 256)
    while e > 64 and cols % e:
        e //= 2
    if cols % e:
        raise ValueError(f"row length {cols} is not a multiple of 64")
    return e


def tile_bytes_for(cols: int, min_tile: int = 1 << 20) -> int:
    """Tile size of a projection's VRN1 frame: the reference's default 1 MiB
    (formats/bf16_rans.py:148), or the next power of two holding 128 rows when
    rows are longer (2 MiB for rows of 6144, config 4's pages), so that a
    block of 128 rows -- the tensor-core kernel's M -- spans at most two tiles."""
    need = 128 * 2 * cols
    t = min_tile
    while t < need:
        t *= 2
    return t


class ProjPage:
    """One expert projection as a resident compressed page."""

    def __init__(self, w_bits: np.ndarray, device, every: int | None = None, frame: bytes | None = None,
                 tile_bytes: int | None = None, stream: torch.cuda.Stream | None = None):
        rows, cols = w_bits.shape
        self.rows, self.cols = int(rows), int(cols)
        every = every or every_for(self.rows, self.cols)
        if frame is None:
            frame, _ = bf16_rans.encode(np.ascontiguousarray(w_bits).view(np.uint8),
                                        tile_bytes=tile_bytes or tile_bytes_for(cols))
        self.page = bf16_rans.RansPage(frame, device=device, every=every, stream=stream)
        if self.page.n_tiles > MAX_TILES:
            raise ValueError(f"a {rows}x{cols} projection in {self.page.n_tiles} tiles: the fused kernels take at "
                             f"most {MAX_TILES} tiles per projection (use larger tiles)")
        self.frame_bytes = len(frame)

    def record(self) -> tuple:
        p = self.page
        return (p.src.data_ptr(), p.tiles.data_ptr(), p.ckpt.data_ptr(), p.ckpt_base.data_ptr(), p.n_tiles,
                p.every, self.rows, self.cols)


class ExpertStore:
    """Compressed gate/up/down pages of E experts and their device page table.

    `experts[e]` is (Wg, Wu, Wd) as BF16 bit arrays, or None for an expert whose
    pages live on another GPU (its table entry has zero tiles, so the fused
    kernels skip it).  `alias` maps an expert id to another expert whose pages it
    shares (tests that route many experts over a few page sets).  Every
    projection is one VRN1 frame with tiles of `tile_bytes` (default
    tile_bytes_for(cols)) and a checkpoint every every_for(rows, cols) symbols.  A
    weight may also be a callable returning the bit array (generated when its
    page is built); `threads` > 1 builds pages concurrently."""

    def __init__(self, experts: list, device, alias: dict[int, int] | None = None, tile_bytes: int | None = None,
                 threads: int = 1):
        self.device = _device.require_cuda(device)
        alias = alias or {}
        self.pages: list = [None] * len(experts)
        todo = [(e, j, w) for e, ws in enumerate(experts) if ws is not None and e not in alias
                for j, w in enumerate(ws)]
        built: dict = {}
        if threads > 1 and len(todo) > 1:
            # encode + index many projections at once: a host thread and a
            # stream each (a page's index build is a small cold decode)
            from concurrent.futures import ThreadPoolExecutor

            local = threading.local()

            def one(item):
                e, j, w = item
                if not hasattr(local, "stream"):
                    local.stream = torch.cuda.Stream(self.device)
                with torch.cuda.stream(local.stream):  # the page's status read-back follows its decode
                    pg = ProjPage(w() if callable(w) else w, self.device, tile_bytes=tile_bytes,
                                  stream=local.stream)
                local.stream.synchronize()
                return (e, j), pg

            with ThreadPoolExecutor(max_workers=threads) as pool:
                built = dict(pool.map(one, todo))
        else:
            for e, j, w in todo:
                built[(e, j)] = ProjPage(w() if callable(w) else w, self.device, tile_bytes=tile_bytes)
        for e, ws in enumerate(experts):
            if ws is not None and e not in alias:
                self.pages[e] = tuple(built[(e, j)] for j in range(3))
        for e, src in alias.items():
            self.pages[e] = self.pages[src]
        first = next(t for t in self.pages if t is not None)
        self.I, self.H = first[0].rows, first[0].cols
        tab = np.zeros(len(self.pages), dtype=PAGES_DTYPE)
        for i, trip in enumerate(self.pages):
            if trip is not None:
                g, u, d = trip
                tab[i] = (g.record(), u.record(), d.record())
        self.table = _device.tensor_from_numpy(tab, self.device)
        present = [t for t in self.pages if t is not None]
        self.local = [e for e, t in enumerate(self.pages) if t is not None]
        self.gate_tiles = max(g.page.n_tiles for g, _, _ in present)
        self.down_tiles = max(d.page.n_tiles for _, _, d in present)
        distinct = {id(t): t for t in present}.values()
        self.compressed_bytes = sum(p.frame_bytes for t in distinct for p in t)
        self.raw_bytes = sum(2 * p.rows * p.cols for t in distinct for p in t)

    def __len__(self) -> int:
        return len(self.pages)


def _variant(family: str, norm_topk: bool, routed_scale: float, shared: int | None,
             shared_gate_w: torch.Tensor | None, router_bias: torch.Tensor | None):
    from .._lib import MOE_FAMILIES, MoeVariant

    if family not in MOE_FAMILIES:
        raise ValueError(f"unknown MoE family {family!r} (one of {sorted(MOE_FAMILIES)})")
    if family == "qwen35":
        norm_topk = True  # qwen35.py:592 always renormalises
    return MoeVariant(MOE_FAMILIES[family], int(norm_topk), float(routed_scale), -1 if shared is None else int(shared),
                      None if shared_gate_w is None else shared_gate_w.data_ptr(),
                      None if router_bias is None else router_bias.data_ptr())


class MoeLayer:
    """Device-side MoE layer (routing on the GPU, no host synchronisation).

    `family` picks the reference layer the math follows: "generic"
    (runtime/layer_runner.py run_moe_mlp), "qwen35" (runtime/qwen35.py _moe:
    zero-centred norm weight, ascending expert order, shared expert gated by
    `shared_gate_w`) or "glm" (runtime/glm.py: fp32 sigmoid router with the
    correction bias `router_bias`, `routed_scale`, fp32 route weights, shared
    expert).  `shared` is the store index of the shared expert (after the
    router's experts), or None."""

    def __init__(self, store: ExpertStore, router_w: torch.Tensor, norm_w: torch.Tensor | None, *,
                 top_k: int, norm_topk: bool = True, eps: float = 1e-6, family: str = "generic",
                 shared: int | None = None, shared_gate_w: torch.Tensor | None = None,
                 router_bias: torch.Tensor | None = None, routed_scale: float = 1.0):
        self.store = store
        self.router_w = router_w.contiguous()
        self.n_experts = int(self.router_w.shape[0])
        self.norm_w = None if norm_w is None else norm_w.contiguous()
        self.top_k = int(top_k)
        self.norm_topk = bool(norm_topk) or family == "qwen35"
        self.eps = float(eps)
        self.family = family
        self.shared = shared
        self.shared_gate_w = None if shared_gate_w is None else shared_gate_w.contiguous()
        self.router_bias = None if router_bias is None else router_bias.float().contiguous()
        self.routed_scale = float(routed_scale)
        self.variant = _variant(family, self.norm_topk, self.routed_scale, shared, self.shared_gate_w,
                                self.router_bias)
        self._scratch: dict[int, torch.Tensor] = {}
        self.status = torch.zeros(1, dtype=torch.int32, device=store.device)

    def scratch(self, T: int) -> torch.Tensor:
        if T not in self._scratch:
            n = load().voom_moe_scratch_bytes_v(ctypes.byref(self.variant), T, self.store.H, self.store.I,
                                                self.top_k)
            self._scratch[T] = torch.empty(int(n), dtype=torch.uint8, device=self.store.device)
        return self._scratch[T]

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None,
                stream: torch.cuda.Stream | None = None, residual: bool = True) -> torch.Tensor:
        """x: (T, H) BF16 on the device -> x + moe(x) (or moe(x)), (T, H) BF16."""
        T, H = x.shape
        x = x.contiguous()
        out = torch.empty_like(x) if out is None else out
        s = self.scratch(T)
        st = self.store
        check(load().voom_moe_layer_v(ctypes.byref(self.variant), st.table.data_ptr(), self.n_experts,
                                      self.router_w.data_ptr(),
                                      None if self.norm_w is None else self.norm_w.data_ptr(), self.eps,
                                      x.data_ptr(), out.data_ptr(), T, H, st.I, self.top_k, st.gate_tiles,
                                      st.down_tiles, int(residual), s.data_ptr(), s.numel(),
                                      self.status.data_ptr(), _device.stream_ptr(st.device, stream)),
              "voom_moe_layer_v")
        return out

    __call__ = forward

    def check_status(self) -> None:
        """Raises ValueError if any forward since the last check met a damaged
        expert page (or a routing overflow); clears the status word.  Forward
        itself never synchronises, so callers check once per step, where they
        read results anyway."""
        raise_on_status(self.status, "MoE layer")


class MoeStepGraph:
    """A fixed stack of MoE layers for T tokens, captured once in a CUDA graph
    and replayed per decode step: one graph launch instead of about eight
    kernel launches per layer, with results bit-identical to calling the
    layers one by one.  `step(x)` copies x into the graph's input buffer,
    replays, and returns the graph's output buffer (overwritten by the next
    step).  Every layer's scratch is allocated before the capture, so the
    replay allocates nothing."""

    def __init__(self, layers: list, T: int, H: int, device, *, residual: bool = True):
        self.layers = list(layers)
        self.T, self.H = int(T), int(H)
        self.device = torch.device(device)
        self.x = torch.zeros((self.T, self.H), dtype=torch.bfloat16, device=self.device)
        self.bufs = [torch.empty_like(self.x) for _ in range(2)]
        for layer in self.layers:
            layer.scratch(self.T)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._run(residual)  # warm-up outside the capture
        torch.cuda.current_stream(self.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self._run(residual)

    def _run(self, residual: bool) -> torch.Tensor:
        cur = self.x
        for i, layer in enumerate(self.layers):
            nxt = self.bufs[i % 2]
            layer(cur, out=nxt, residual=residual)
            cur = nxt
        return cur

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.out

    def step(self, x: torch.Tensor) -> torch.Tensor:
        self.x.copy_(x)
        return self.replay()

    def check_status(self) -> None:
        """check_status() of every layer of the stack (one synchronisation)."""
        for i, layer in enumerate(self.layers):
            raise_on_status(layer.status, f"MoE layer {i}")


def route_rows(idx: np.ndarray):
    """Host mirror of the device route plan: unique experts in first-appearance
    order over (position, slot), tokens per expert, route-row offsets, the token
    of every route row, and each token's rows ordered by that expert order (the
    order runtime/layer_runner.py:387-394 accumulates contributions in)."""
    T, k = idx.shape
    order: list[int] = []
    rows: dict[int, list[int]] = {}
    for p in range(T * k):
        e = int(idx[p // k, p % k])
        if e not in rows:
            order.append(e)
            rows[e] = []
        rows[e].append(p // k)
    ntok = [len(rows[e]) for e in order]
    uoff = np.concatenate([[0], np.cumsum(ntok)]).astype(np.int64)
    upair = [t for e in order for t in rows[e]]
    tok_order = [[q for u in range(len(order)) for q in range(uoff[u], uoff[u + 1]) if upair[q] == t]
                 for t in range(T)]
    return order, ntok, uoff, upair, tok_order


def zipf_popularity(n_experts: int, s: float = 1.1, seed: int = 0) -> np.ndarray:
    """Expert popularity Zipf(s) over ranks, assigned to experts by a seeded permutation."""
    w = 1.0 / np.arange(1, n_experts + 1, dtype=np.float64) ** s
    perm = np.random.default_rng(seed).permutation(n_experts)
    p = np.empty(n_experts)
    p[perm] = w / w.sum()
    return p


def place_experts(load, world: int) -> list[list[int]]:
    """Longest-processing-time placement: experts by descending expected load,
    each to the currently least-loaded rank.  Returns the experts of each rank."""
    load = np.asarray(load, dtype=np.float64)
    bins = [[] for _ in range(world)]
    tot = np.zeros(world)
    for e in sorted(range(load.size), key=lambda i: (-load[i], i)):
        r = int(np.argmin(tot))
        bins[r].append(e)
        tot[r] += load[e]
    return [sorted(b) for b in bins]


PAGE_LOAD = 16  # load of one expert's page decode, in tokens (kPageLoad in csrc/expert.cu)


def assign_owners(unit_experts, ntok, holders, world: int) -> list[int]:
    """Owner rank of each unique expert under expert parallelism, as
    moe_route_owners computes it on the device: an expert one rank holds is
    that rank's; the others, in unique order after all single-holder experts
    are counted, go to their least loaded holder (lowest rank on a tie); load
    of a unique expert = PAGE_LOAD + its tokens.  `holders[e]`: bit r = rank r
    holds expert e.  An expert no rank holds gets `world` (computed nowhere)."""
    mask = (1 << world) - 1
    load = [0] * world
    owner = [world] * len(unit_experts)
    for u, e in enumerate(unit_experts):
        h = int(holders[e]) & mask
        if h and not h & (h - 1):
            owner[u] = h.bit_length() - 1
            load[owner[u]] += PAGE_LOAD + int(ntok[u])
    for u, e in enumerate(unit_experts):
        h = int(holders[e]) & mask
        if not h or not h & (h - 1):
            continue
        best = min((o for o in range(world) if h >> o & 1), key=lambda o: (load[o], o))
        owner[u] = best
        load[best] += PAGE_LOAD + int(ntok[u])
    return owner


def holders_for(placement: list[list[int]], n_entries: int, replicated=()) -> np.ndarray:
    """Holder masks (bit r = rank r holds the expert) from per-rank expert
    lists, with the `replicated` experts held by every rank."""
    h = np.zeros(n_entries, dtype=np.uint32)
    for r, experts in enumerate(placement):
        for e in experts:
            h[e] |= np.uint32(1 << r)
    for e in replicated:
        h[e] = np.uint32((1 << len(placement)) - 1)
    return h


class ExpertParallelMoeLayer:
    """MoE layer with experts spread over the ranks of a process group (NCCL).

    Every rank routes all tokens (replicated router) and computes only the
    routed experts it owns: an expert whose pages one rank holds is that
    rank's; an expert several ranks hold (replicated hot experts) goes to the
    least loaded of its holders by a rule every rank evaluates alike on the
    device, so each route row is computed exactly once and only owned experts
    launch work.  The route rows come back in token-major order; a
    reduce-scatter over tokens (every row has one nonzero contributor, so the
    sum is exact) gives each rank the rows of its share of the tokens, the
    rank applies the ordered combine to them, and an all-gather of the
    combined rows gives every rank the layer output -- bit-identical to
    MoeLayer on one GPU, for about (1 + 1/rows_per_token) / 2 of the bytes an
    all-reduce of the route rows would move.

    Which ranks hold which experts is gathered once at construction from the
    ranks' stores (`holders`, one bit mask per store entry, overrides it; with
    `rank` and `world` it lets one process emulate a rank).  Same family
    options as MoeLayer."""

    def __init__(self, store: ExpertStore, router_w: torch.Tensor, norm_w: torch.Tensor | None, *, top_k: int,
                 norm_topk: bool = True, eps: float = 1e-6, group=None, router_bias: torch.Tensor | None = None,
                 family: str = "generic", shared: int | None = None, shared_gate_w: torch.Tensor | None = None,
                 routed_scale: float = 1.0, holders: np.ndarray | None = None, rank: int | None = None,
                 world: int | None = None):
        import torch.distributed as dist

        from .._lib import MoeEp

        self.store = store
        self.router_w = router_w.contiguous()
        self.n_experts = int(self.router_w.shape[0])
        self.router_bias = None if router_bias is None else router_bias.float().contiguous()
        self.norm_w = None if norm_w is None else norm_w.contiguous()
        self.top_k = int(top_k)
        self.norm_topk = bool(norm_topk) or family == "qwen35"
        self.eps = float(eps)
        self.group = group
        self.shared = shared
        self.shared_gate_w = None if shared_gate_w is None else shared_gate_w.contiguous()
        self.variant = _variant(family, self.norm_topk, routed_scale, shared, self.shared_gate_w, self.router_bias)
        self.rows_per_token = self.top_k + (0 if shared is None else 1)
        on = dist.is_available() and dist.is_initialized()
        self.world = int(world) if world is not None else (dist.get_world_size(group) if on else 1)
        self.rank = int(rank) if rank is not None else (dist.get_rank(group) if on else 0)
        if not 0 <= self.rank < self.world <= 32:
            raise ValueError(f"rank {self.rank} of {self.world}: expert parallelism takes 1..32 ranks")
        if holders is None:
            mine = torch.zeros(len(store), dtype=torch.int64, device=store.device)
            if store.local:
                mine[torch.tensor(store.local, device=store.device)] = 1 << self.rank
            if self.world > 1:
                dist.all_reduce(mine, group=group)  # distinct bits: the sum is the OR
            holders = mine.cpu().numpy()
        holders = np.asarray(holders, dtype=np.int64).astype(np.uint32)
        if holders.shape != (len(store),):
            raise ValueError(f"holders: one mask per store entry ({len(store)}), got {holders.shape}")
        self.holders = _device.tensor_from_numpy(holders, store.device)
        self._ep = {}
        self._MoeEp = MoeEp
        self._scratch: dict[int, torch.Tensor] = {}
        self._bufs: dict[int, tuple] = {}
        self.status = torch.zeros(1, dtype=torch.int32, device=store.device)
        self.last_collective_bytes = 0

    def t_pad(self, T: int) -> int:
        return -(-T // self.world) * self.world

    def buffers(self, T: int) -> tuple:
        """(scratch, token-major rows, this rank's rows, this rank's combined
        rows, combined rows of all ranks) for T tokens, allocated once."""
        st = self.store
        if T not in self._scratch:
            n = load().voom_moe_scratch_bytes_v(ctypes.byref(self.variant), T, st.H, st.I, self.top_k)
            self._scratch[T] = torch.empty(int(n), dtype=torch.uint8, device=st.device)
            tp = self.t_pad(T)
            ts = tp // self.world
            self._bufs[T] = (torch.empty((tp * self.rows_per_token, st.H), dtype=torch.bfloat16, device=st.device),
                             torch.empty((ts * self.rows_per_token, st.H), dtype=torch.bfloat16, device=st.device),
                             torch.empty((ts, st.H), dtype=torch.bfloat16, device=st.device),
                             torch.empty((tp, st.H), dtype=torch.bfloat16, device=st.device))
            self._ep[T] = self._MoeEp(self.holders.data_ptr(), self.rank, self.world, tp)
        return (self._scratch[T], *self._bufs[T])

    def experts(self, x: torch.Tensor) -> torch.Tensor:
        """Phase 1 on this rank: routes + this rank's route rows, token-major
        (t_pad(T) * rows_per_token rows; other ranks' rows zero)."""
        T, H = x.shape
        st = self.store
        s, y_tm = self.buffers(T)[:2]
        check(load().voom_moe_experts_ep(ctypes.byref(self.variant), ctypes.byref(self._ep[T]), st.table.data_ptr(),
                                         self.n_experts, self.router_w.data_ptr(),
                                         None if self.norm_w is None else self.norm_w.data_ptr(), self.eps,
                                         x.data_ptr(), T, H, st.I, self.top_k, st.gate_tiles, st.down_tiles,
                                         y_tm.data_ptr(), s.data_ptr(), s.numel(), self.status.data_ptr(),
                                         _device.stream_ptr(st.device, None)), "voom_moe_experts_ep")
        return y_tm

    def combine(self, x: torch.Tensor, rows: torch.Tensor, out: torch.Tensor, t0: int, count: int,
                residual: bool = True) -> None:
        """Phase 2: the ordered combine of tokens [t0, t0 + count) from their
        token-major rows into `out` (count rows)."""
        T, H = x.shape
        s = self.buffers(T)[0]
        check(load().voom_moe_combine_tm(s.data_ptr(), rows.data_ptr(), x.data_ptr(), out.data_ptr(), t0, count, H,
                                         int(residual), _device.stream_ptr(self.store.device, None)),
              "voom_moe_combine_tm")

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None, residual: bool = True) -> torch.Tensor:
        import torch.distributed as dist

        x = x.contiguous()
        T, H = x.shape
        out = torch.empty_like(x) if out is None else out
        if self.world == 1:  # one rank: the fused single-GPU layer (no owners, no exchange)
            s = self.buffers(T)[0]
            st = self.store
            check(load().voom_moe_layer_v(ctypes.byref(self.variant), st.table.data_ptr(), self.n_experts,
                                          self.router_w.data_ptr(),
                                          None if self.norm_w is None else self.norm_w.data_ptr(), self.eps,
                                          x.data_ptr(), out.data_ptr(), T, H, st.I, self.top_k, st.gate_tiles,
                                          st.down_tiles, int(residual), s.data_ptr(), s.numel(),
                                          self.status.data_ptr(), _device.stream_ptr(st.device, None)),
                  "voom_moe_layer_v")
            self.last_collective_bytes = 0
            return out
        y_tm = self.experts(x)
        _, _, shard, part, full = self.buffers(T)
        ts = self.t_pad(T) // self.world
        if self.world > 1:
            dist.reduce_scatter_tensor(shard, y_tm, group=self.group)
            self.combine(x, shard, part, self.rank * ts, ts, residual)
            dist.all_gather_into_tensor(full, part, group=self.group)
            self.last_collective_bytes = (y_tm.numel() + full.numel()) * 2
        else:
            self.combine(x, y_tm, full, 0, ts, residual)
            self.last_collective_bytes = 0
        out.copy_(full[:T])
        return out

    __call__ = forward

    def check_status(self) -> None:
        """As MoeLayer.check_status (this rank's experts only)."""
        raise_on_status(self.status, "expert-parallel MoE layer")


def swiglu_grouped(store: ExpertStore, expert_ids: list[int], token_lists: list[list[int]], h: torch.Tensor,
                   stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """Experts grouped on the host: returns y (sum(len(tokens)), H) BF16, rows in
    (expert, token) order, unweighted -- what `_swiglu(h[:, pos], experts[e])`
    yields for each expert of a consume_expert_batches batch."""
    dev = store.device
    ntok = np.array([len(t) for t in token_lists], dtype=np.uint32)
    upair = np.concatenate([np.asarray(t, dtype=np.uint32) for t in token_lists])
    n_rows = int(upair.size)
    T = int(h.shape[0])
    d_ids = _device.tensor_from_numpy(np.asarray(expert_ids, dtype=np.uint32), dev)
    d_ntok = _device.tensor_from_numpy(ntok, dev)
    d_upair = _device.tensor_from_numpy(upair, dev)
    y = torch.empty((n_rows, store.H), dtype=torch.bfloat16, device=dev)
    need = int(load().voom_moe_scratch_bytes(n_rows, store.H, store.I, 1))
    scratch = torch.empty(need, dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    check(load().voom_expert_swiglu(store.table.data_ptr(), d_ids.data_ptr(), len(expert_ids), d_ntok.data_ptr(),
                                    d_upair.data_ptr(), n_rows, T, h.contiguous().data_ptr(), store.H, store.I,
                                    store.gate_tiles, store.down_tiles, y.data_ptr(), scratch.data_ptr(), need,
                                    status.data_ptr(), _device.stream_ptr(dev, stream)), "voom_expert_swiglu")
    raise_on_status(status, "voom_expert_swiglu")
    return y
