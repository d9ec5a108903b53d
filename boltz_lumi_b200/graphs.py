"""CUDA-graph replay of a repeated step (the diffusion score model).

The 200-step diffusion loop calls the same score-model forward with new
coordinates and time each step and the same conditioning, features and token
bias every time.  At small token counts that forward is launch-bound: its
kernels take a few microseconds each and the eager host path between them
takes longer.  :class:`GraphedStep` runs such a callable as a captured CUDA
graph:

* call 1 runs eagerly and records which tensor arguments were passed;
* call 2 compares: argument slots whose tensor changed are *dynamic* (they
  get a graph-owned buffer, refreshed by one device copy per replay), slots
  passing the same tensor again are *constant* (the graph reads that tensor
  in place; a reference is held so its memory stays valid).  It then warms up
  on a side stream and captures;
* later calls with the same structure replay the graph; a constant slot that
  now passes a different tensor, or a different shape / dtype / stride
  anywhere, falls back to an eager call and a capture for the new signature.

Outputs are returned as clones (the graph's own output buffers are rewritten
by the next replay).  The callable must be capture-safe: no host
synchronisation, no data-dependent shapes, no RNG.  All kernels of this
package are (their one-time setup runs in the eager calls).
"""

import torch


def _flatten(obj, leaves):
    """Tensor leaves of nested tuples / lists / dicts, with a hashable structure."""
    if isinstance(obj, torch.Tensor):
        leaves.append(obj)
        return ("T", tuple(obj.shape), obj.dtype, tuple(obj.stride()), obj.device)
    if isinstance(obj, (list, tuple)):
        return (type(obj).__name__, tuple(_flatten(x, leaves) for x in obj))
    if isinstance(obj, dict):
        return ("dict", tuple((k, _flatten(obj[k], leaves)) for k in sorted(obj, key=repr)))
    try:
        hash(obj)
    except TypeError:
        return ("id", id(obj))  # e.g. a callable passed through: identity
    return ("v", obj)


def _rebuild(obj, leaves, it):
    if isinstance(obj, torch.Tensor):
        return leaves[next(it)]
    if isinstance(obj, tuple):
        return tuple(_rebuild(x, leaves, it) for x in obj)
    if isinstance(obj, list):
        return [_rebuild(x, leaves, it) for x in obj]
    if isinstance(obj, dict):  # same key order as _flatten
        return {k: _rebuild(obj[k], leaves, it) for k in sorted(obj, key=repr)}
    return obj


def _clone_out(obj):
    if isinstance(obj, torch.Tensor):
        return obj.clone()
    if isinstance(obj, tuple):
        return tuple(_clone_out(x) for x in obj)
    if isinstance(obj, list):
        return [_clone_out(x) for x in obj]
    if isinstance(obj, dict):
        return {k: _clone_out(v) for k, v in obj.items()}
    return obj


class _Entry:
    def __init__(self, graph, static_leaves, dynamic, output):
        self.graph, self.static_leaves, self.dynamic, self.output = graph, static_leaves, dynamic, output


class GraphedStep:
    """Replay ``fn(*args, **kwargs)`` from a CUDA graph once it repeats.

    ``max_graphs`` bounds how many signatures stay captured (oldest dropped).
    ``stats`` counts eager calls, captures and replays.
    """

    def __init__(self, fn, max_graphs=2, warmup=2):
        self.fn, self.max_graphs, self.warmup = fn, max_graphs, warmup
        self.entries = {}  # structure key -> _Entry
        self.pending = {}  # structure key -> leaf tensors of the first call
        self.pool = None
        self.stats = dict(eager=0, captures=0, replays=0)

    def _eager(self, args, kwargs):
        self.stats["eager"] += 1
        return self.fn(*args, **kwargs)

    def __call__(self, *args, **kwargs):
        leaves = []
        structure = _flatten((args, kwargs), leaves)
        entry = self.entries.get(structure)
        if entry is not None:
            for i, (leaf, static) in enumerate(zip(leaves, entry.static_leaves)):
                if i in entry.dynamic:
                    if leaf is not static:
                        static.copy_(leaf)
                elif leaf is not static:  # a constant slot changed: recapture for the new inputs
                    del self.entries[structure]
                    self.pending[structure] = leaves
                    return self._eager(args, kwargs)
            entry.graph.replay()
            self.stats["replays"] += 1
            return _clone_out(entry.output)
        first = self.pending.pop(structure, None)
        if first is None:
            while len(self.pending) >= 4:  # signatures seen once and never again
                self.pending.pop(next(iter(self.pending)))
            self.pending[structure] = leaves
            return self._eager(args, kwargs)
        dynamic = {i for i, (a, b) in enumerate(zip(leaves, first)) if a is not b}
        static_leaves = [leaf.clone() if i in dynamic else leaf for i, leaf in enumerate(leaves)]
        static_args, static_kwargs = _rebuild((args, kwargs), static_leaves, iter(range(len(static_leaves))))
        entry = self._capture(static_args, static_kwargs, static_leaves, dynamic)
        while len(self.entries) >= self.max_graphs:
            self.entries.pop(next(iter(self.entries)))
        self.entries[structure] = entry
        entry.graph.replay()
        self.stats["replays"] += 1
        return _clone_out(entry.output)

    def _capture(self, args, kwargs, static_leaves, dynamic):
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(self.warmup):  # allocator, library handles and lazy setup outside the capture
                self.fn(*args, **kwargs)
        torch.cuda.current_stream().wait_stream(stream)
        if self.pool is None:
            self.pool = torch.cuda.graph_pool_handle()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, pool=self.pool):
            output = self.fn(*args, **kwargs)
        self.stats["captures"] += 1
        return _Entry(graph, static_leaves, dynamic, output)

    def reset(self):
        """Drop every captured graph (and the tensors they hold)."""
        self.entries.clear()
        self.pending.clear()
