"""CUDA-graph capture of a training step through the CUDA path.

The benchmarks replay the config-2 / config-5 training steps from a captured
CUDA graph; every op on the path (the tcgen05 GEMM, the scans, packing) must
be capture-safe: no host synchronisation, launches on the current stream,
allocations from torch. Replaying the captured step must update the
parameters exactly as the eager step does.
"""

from __future__ import annotations

import pytest
import torch

import myelin_b200 as mb

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _model(dtype, sizes, seed):
    torch.manual_seed(seed)
    params = mb.LIFParams(tau_mem=20.0, threshold=1.0)
    layers = [mb.LinearSurrogateLIF(fi, fo, params, surrogate=mb.superspike_surrogate,
                                    surrogate_slope=10.0, stream_synapse=True)
              for fi, fo in zip(sizes[:-2], sizes[1:-1])]
    layers.append(mb.LinearSurrogateLIFRate(sizes[-2], sizes[-1], params,
                                            surrogate=mb.superspike_surrogate,
                                            surrogate_slope=10.0, reduction="none"))
    return torch.nn.Sequential(*layers).to(DEV, dtype)


@pytest.mark.parametrize("dtype,sizes", [(torch.float32, (64, 96, 10)),
                                         (torch.bfloat16, (256, 512, 512, 10))])
def test_graph_replay_matches_eager_training(dtype, sizes):
    g = torch.Generator(device=DEV).manual_seed(1)
    x = (torch.rand((20, 32, sizes[0]), generator=g, device=DEV) < 0.2).to(dtype)
    target = torch.rand((32, sizes[-1]), generator=g, device=DEV) * 0.3

    def make():
        model = _model(dtype, sizes, seed=3)
        opt = torch.optim.SGD(model.parameters(), lr=0.5)

        def step():
            opt.zero_grad(set_to_none=True)
            loss = torch.nn.functional.mse_loss(model(x).float(), target)
            loss.backward()
            opt.step()
            return loss

        return model, step

    eager_model, eager_step = make()
    for _ in range(4):
        eager_step()

    graph_model, graph_step = make()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        graph_step()  # warm-up step (also the first training step)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        graph_step()  # recorded, not run: 1 warm-up + 3 replays = 4 steps
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    for pe, pg in zip(eager_model.parameters(), graph_model.parameters()):
        assert torch.equal(pe, pg)
