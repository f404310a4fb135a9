"""CUDA Graph capture of the whole block (reference: block_benchmark.py:48-64)."""

import torch


@torch.inference_mode()
def capture_forward(block, x):
    """Warm up on a side stream, capture block(x), replay once and check it
    against eager output (rtol = atol = 0.03, as the reference does)."""
    expected = block(x).clone()
    stream = torch.cuda.Stream(device=x.device)
    stream.wait_stream(torch.cuda.current_stream(x.device))
    with torch.cuda.stream(stream):
        for _ in range(3):
            block(x)
    torch.cuda.current_stream(x.device).wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        output = block(x)
    graph.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(output, expected, rtol=0.03, atol=0.03)
    return graph, output
