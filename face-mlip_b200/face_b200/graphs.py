"""One energy+force evaluation on a fixed neighbour graph as a CUDA-graph replay.

An evaluation on a fixed graph reads nothing back from the device (face_b200.ops keeps each structure's PME data on
the host from graph construction), and every library kernel launches on torch's current stream, so the forward, the
autograd backward and all their launches can be captured once and replayed: a replay costs one launch on the host
instead of the ~300-500 of an eager evaluation, which is what bounds small systems (molecule batches, MD of a few
thousand atoms).  The reference has no counterpart (it runs eagerly; face/model.py:689 only avoids one sync).

    ev = GraphedEvaluation(model, graph)         # captures after warm-up (weights packed, FFT plans made)
    out = ev(pos)                                 # copies pos into the captured input, replays
    out["energy"], out["atom_energy"], out["forces"]   # tensors owned by the capture, overwritten by each replay

The captured graph is valid for the neighbour list it was captured with (the calculator recaptures after each
rebuild) and for the model's weights at capture time.
"""
import torch

from . import _lib, ops


class GraphedEvaluation:
    def __init__(self, model, graph, warmup=2):
        self.model = model
        self.pos = graph["pos"].detach().clone().requires_grad_(True)      # the captured input
        self.graph_dict = dict(graph, pos=self.pos)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):                  # warm-up off the capture: caches, plans, packed weights
            for _ in range(warmup):
                self._evaluate()
        torch.cuda.current_stream().wait_stream(side)
        self.cuda_graph = torch.cuda.CUDAGraph()
        counting, calls = _lib.COUNTING, dict(_lib.CALLS)
        _lib.CALLS.clear()
        _lib.COUNTING = True
        try:
            with torch.cuda.graph(self.cuda_graph):
                self.out = self._evaluate()
        finally:
            self.launches = _lib.launches()            # library kernels in one replay
            _lib.CALLS.clear()
            _lib.CALLS.update(calls)
            _lib.COUNTING = counting

    def _evaluate(self):
        return ops.face_forward(self.model, self.graph_dict, forces=True)

    def __call__(self, pos):
        with torch.no_grad():
            self.pos.copy_(pos)
        self.cuda_graph.replay()
        return self.out
