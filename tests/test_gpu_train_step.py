"""A whole training step with the uDTW loss captured in one CUDA graph (B200).

The step (forecaster, sigma network, uDTW loss through the native kernels,
backward, Adam) is launch-bound at the batch sizes of the reference's ECG5000
experiment, so it is meant to run as a graph replay.  The native ops launch
on the caller's current stream and take their scratch from the caching
allocator, so they can be captured.  The replayed losses must follow the eager
trajectory of the same model.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tw():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import torchwarp_b200
    return torchwarp_b200


def _setup(tw, dev):
    torch.manual_seed(7)
    f = torch.nn.Sequential(torch.nn.Linear(84, 128), torch.nn.ReLU(),
                            torch.nn.Linear(128, 56)).to(dev)
    s = torch.nn.Sequential(torch.nn.Linear(56, 32), torch.nn.ReLU(),
                            torch.nn.Linear(32, 56)).to(dev)
    opt = torch.optim.Adam(list(f.parameters()) + list(s.parameters()), lr=1e-3,
                           capturable=True)
    crit = tw.UDTW(gamma=0.1, beta=0.01)

    def step(x, y):
        pred = f(x)
        sig = lambda v: 2.0 * torch.sigmoid(s(v)) + 0.1  # noqa: E731
        d, p = crit(pred.unsqueeze(-1), y.unsqueeze(-1), sig(pred).unsqueeze(-1),
                    sig(y).unsqueeze(-1))
        loss = (d + p).mean()
        opt.zero_grad(set_to_none=False)
        loss.backward()
        opt.step()
        return loss

    return step


def test_graph_captured_step_matches_eager(tw):
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(11)
    data = torch.randn(400, 140, device=dev, generator=g)
    batches = [(data[k * 50:(k + 1) * 50, :84], data[k * 50:(k + 1) * 50, 84:]) for k in range(8)]

    step = _setup(tw, dev)
    eager = [step(x, y).item() for x, y in batches]

    step = _setup(tw, dev)
    sx, sy = torch.empty(50, 84, device=dev), torch.empty(50, 56, device=dev)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for x, y in batches[:3]:
            sx.copy_(x)
            sy.copy_(y)
            step(sx, sy)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        loss = step(sx, sy)
    replayed = []
    for x, y in batches[3:]:
        sx.copy_(x)
        sy.copy_(y)
        graph.replay()
        replayed.append(loss.item())
    for a, b in zip(replayed, eager[3:]):
        assert abs(a - b) <= 1e-4 * abs(b), (replayed, eager[3:])
    assert tw._native.lib().tw_device_error() == 0
