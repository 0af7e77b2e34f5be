"""Standalone CUDA Graph owner: stable pointers, replayed plan, layer-private scratch.

Same lifecycle as the reference's ``runtime/graph.py:6-79`` (``update`` with host
capacity checks -> ``capture`` after warm-ups -> ``replay`` with ready/done events),
extended to CSR KV (``csr=True``): each layer then owns an ``indptr`` [Bcap+1] and a
``kv_indices`` buffer of ``index_capacity`` slots instead of a page table.  The plan
is rebuilt inside the graph on every replay and shared by all layers.
"""
import torch

from .engine import DecodeEngine


class DecodeGraph:
    def __init__(self, engine: DecodeEngine, keys, kv_pairs, *, csr=False, index_capacity=None):
        if len(keys) != len(engine.layers) or len(kv_pairs) != len(keys):
            raise ValueError("one key and KV pair per layer required")
        if not keys or any(key != keys[0] for key in keys):
            raise ValueError("incompatible layers require separate plan/graph instances")
        self.engine, self.kv_pairs, self.csr = engine, kv_pairs, csr
        c, p = engine.config, engine.plan
        self.q = [torch.empty_like(layer.output) for layer in engine.layers]
        if csr:
            if c.page_size != 1:
                raise ValueError("CSR graphs use one-token pages")
            cap = index_capacity or c.batch_capacity * c.max_context
            self.index_capacity = cap
            self.indptr = torch.zeros(c.batch_capacity + 1, dtype=torch.int32, device=p.device)
            self.pages = [torch.zeros(cap, dtype=torch.int32, device=p.device) for _ in keys]
        else:
            self.indptr = None
            self.pages = [torch.zeros((c.batch_capacity, c.max_pages), dtype=torch.int32,
                                      device=p.device) for _ in keys]
        self.ready, self.done = torch.cuda.Event(), torch.cuda.Event()
        self.graph = None
        self.has_run = False

    def update(self, queries, page_tables, lengths, splits):
        """Host lengths are already known by the scheduler; no GPU scalar readback.

        Paged: ``page_tables[i]`` is [n, max_pages].  CSR: ``page_tables[i]`` is the
        layer's flat kv_indices (request-major, sum(lengths) entries).
        """
        c, p = self.engine.config, self.engine.plan
        if not 0 < len(lengths) <= c.batch_capacity or len(splits) != len(lengths):
            raise ValueError("choose a larger graph or upstream before submitting")
        if any(x < 0 or x > c.max_context for x in lengths):
            raise ValueError("context outside graph capacity")
        if any(x < 1 or x > c.max_splits for x in splits):
            raise ValueError("split capacity exceeded")
        if len(queries) != len(self.q) or len(page_tables) != len(self.pages):
            raise ValueError("layer count mismatch")
        n = len(lengths)
        total = sum(lengths)
        for q, pages in zip(queries, page_tables):
            if tuple(q.shape) != (n, c.query_heads, c.head_dim):
                raise ValueError("input shape mismatch")
            if self.csr:
                if pages.ndim != 1 or pages.numel() != total or total > self.index_capacity:
                    raise ValueError("kv_indices must hold sum(lengths) <= index_capacity entries")
            elif tuple(pages.shape) != (n, c.max_pages):
                raise ValueError("input shape mismatch")
        stream = torch.cuda.current_stream(p.device)
        if self.has_run:
            stream.wait_event(self.done)
        p.lengths.zero_()
        p.splits.fill_(1)
        p.lengths[:n].copy_(torch.tensor(lengths, dtype=torch.int32), non_blocking=False)
        p.splits[:n].copy_(torch.tensor(splits, dtype=torch.int32), non_blocking=False)
        p.active.fill_(n)
        if self.csr:
            pointers = [0]
            for x in lengths:
                pointers.append(pointers[-1] + x)
            self.indptr[:n + 1].copy_(torch.tensor(pointers, dtype=torch.int32))
        for target_q, target_pages, q, pages in zip(self.q, self.pages, queries, page_tables):
            target_q[:n].copy_(q)
            if self.csr:
                target_pages[:total].copy_(pages)
            else:
                target_pages[:n].copy_(pages)
        self.ready.record(stream)

    def _step(self):
        self.engine.prepare()
        for i, (k, v) in enumerate(self.kv_pairs):
            self.engine.execute(self.q[i], k, v, self.pages[i], layer=i, indptr=self.indptr)

    def capture(self, warmup=3):
        """Explicit opt-in GPU operation. Never invoked at import or installation."""
        if self.graph is not None:
            raise RuntimeError("capture once; create another instance to change geometry")
        stream = torch.cuda.Stream(device=self.engine.plan.device)
        stream.wait_event(self.ready)
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                self._step()
        stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self._step()
        self.done.record(stream)
        self.has_run = True

    def replay(self):
        if self.graph is None:
            raise RuntimeError("capture after initializing representative inputs")
        stream = torch.cuda.current_stream(self.engine.plan.device)
        stream.wait_event(self.ready)
        if self.has_run:
            stream.wait_event(self.done)
        self.graph.replay()
        self.done.record(stream)
        self.has_run = True
        return [layer.output for layer in self.engine.layers]
