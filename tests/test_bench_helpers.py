"""bench.py helpers that need no GPU: the step-graph kernel count degrades to None (the bench
then reports its lower bound) instead of raising when a graph cannot be inspected."""
import bench


class _NoGraph:
    def raw_cuda_graph(self):
        raise RuntimeError("keep_graph was not set")


def test_graph_kernels_returns_none_when_not_inspectable():
    assert bench.graph_kernels(_NoGraph()) is None
    assert bench.graph_kernels(object()) is None
