"""bench.py counts its own kernel launches from the captured step graph (``graph_kernels``):
one decode GEMM captured alone is one libw4 kernel node and nothing else."""
import pytest
import torch

import bench
from xe2x2_b200 import ops, synth

pytestmark = pytest.mark.gpu


def test_graph_kernels_counts_one_decode_gemm(cuda):
    K, N, gs = 1024, 1024, 128
    qw, qz, sc, _ = synth.gptq_weights(K, N, gs, asym=True, seed=3, device=cuda)
    a = synth.activations(1, K, torch.bfloat16, seed=4, device=cuda)
    out = torch.empty((1, N), dtype=torch.bfloat16, device=cuda)
    ops.gptq_gemm(a, qw, qz, sc, gs, 1, out=out)  # modules loaded outside the capture
    torch.cuda.synchronize()
    st = torch.cuda.Stream(cuda)
    st.wait_stream(torch.cuda.current_stream(cuda))
    g = torch.cuda.CUDAGraph(keep_graph=True)
    with torch.cuda.stream(st):
        ops.gptq_gemm(a, qw, qz, sc, gs, 1, out=out)  # this stream's workspace exists before capture
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=st):
            ops.gptq_gemm(a, qw, qz, sc, gs, 1, out=out)
    torch.cuda.current_stream(cuda).wait_stream(st)
    counts = bench.graph_kernels(g)
    assert counts == {"w4": 1, "nccl": 0, "other": 0}, counts
    g.instantiate()
    g.replay()
    torch.cuda.synchronize()
