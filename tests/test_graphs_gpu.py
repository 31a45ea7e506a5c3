"""The operators inside a captured CUDA graph: one graph holding a persistent
causal bf16 attention launch (counter-based work units), an fp16 D = 64
attention, the fp32 split-precision path (staging kernel + programmatic
dependent launch) and the MLP block is replayed several times in one stream,
and every replay must equal the eager results bit for bit."""

import pytest
import torch

from cs348k_fast_attention_grammar_b200 import attention, device_status, mlp

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _rand(shape, seed, dtype, amp=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * amp).to(dtype).to(DEV)


def test_graph_capture_and_replay_matches_eager():
    q, k, v = (_rand((1, 160, 512, 128), 500 + i, torch.bfloat16) for i in range(3))
    qh, kh, vh = (_rand((2, 3, 700, 64), 510 + i, torch.float16) for i in range(3))
    qf, kf, vf = (_rand((1, 2, 300, 64), 520 + i, torch.float32) for i in range(3))
    x = _rand((512, 256), 530, torch.bfloat16)
    w1 = _rand((256, 1024), 531, torch.bfloat16, amp=256 ** -0.5)
    w2 = _rand((1024, 256), 532, torch.bfloat16, amp=1024 ** -0.5)

    want = [attention(q, k, v, causal=True), attention(qh, kh, vh),
            attention(qf, kf, vf, causal=True, precise=True), mlp(x, w1, w2)]
    torch.cuda.synchronize()

    outs = [torch.empty_like(w) for w in want]
    hidden = torch.empty((512, 1024), dtype=torch.bfloat16, device=DEV)

    def step():
        attention(q, k, v, causal=True, out=outs[0])
        attention(qh, kh, vh, out=outs[1])
        attention(qf, kf, vf, causal=True, precise=True, out=outs[2])
        mlp(x, w1, w2, hidden=hidden, out=outs[3])

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()                                  # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        step()
    for _ in range(5):
        for o in outs:
            o.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        for o, w in zip(outs, want):
            assert torch.equal(o, w)
    assert device_status() == 0
