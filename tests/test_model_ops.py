"""Full-model decode driver: the fused elementwise steps against torch fp32
references, and a small decoder whose CUDA-graph decode matches its eager decode
token for token (same kernels, device-side counters, graph capture restores the
host counters)."""

import pytest
import torch

from qevict_b200 import _native as N

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def bf(x):
    return x.to(torch.bfloat16).float()


@pytest.mark.parametrize("rows,cols,with_delta", [(1, 4096, True), (3, 4096, False), (2, 1032, True)])
def test_add_rmsnorm(rows, cols, with_delta):
    g = torch.Generator(device="cuda").manual_seed(rows + cols)
    x = torch.randn(rows, cols, generator=g, device="cuda").to(torch.bfloat16)
    d = torch.randn(rows, cols, generator=g, device="cuda").to(torch.bfloat16) if with_delta else None
    w = (1 + 0.1 * torch.randn(cols, generator=g, device="cuda")).to(torch.bfloat16)
    h = torch.empty_like(x)
    xs = bf(x + d) if with_delta else x.float()
    rc = N.lib().qv_add_rmsnorm(rows, cols, N.ptr(x), N.ptr(d), N.ptr(w), 1e-5, N.ptr(h),
                                torch.cuda.current_stream().cuda_stream)
    N.check(rc, "qv_add_rmsnorm")
    assert torch.equal(x.float(), xs)                       # the residual add, rounded once
    ref = xs * torch.rsqrt((xs * xs).mean(-1, keepdim=True) + 1e-5) * w.float()
    err = (h.float() - bf(ref)).abs()
    assert bool((err <= bf(ref).abs() * 2.0 ** -7 + 1e-6).all())   # one bf16 ulp


def test_silu_mul():
    g = torch.Generator(device="cuda").manual_seed(3)
    gu = (torch.randn(2, 2 * 14336, generator=g, device="cuda") * 3).to(torch.bfloat16)
    out = torch.empty(2, 14336, dtype=torch.bfloat16, device="cuda")
    rc = N.lib().qv_silu_mul(2, 14336, N.ptr(gu), N.ptr(out), torch.cuda.current_stream().cuda_stream)
    N.check(rc, "qv_silu_mul")
    gg, u = gu.float()[:, :14336], gu.float()[:, 14336:]
    ref = bf(bf(gg / (1 + torch.exp(-gg))) * u)
    err = (out.float() - ref).abs()
    assert bool((err <= ref.abs() * 2.0 ** -7 + 1e-6).all())


@pytest.mark.parametrize("side_fold", [False, True])
def test_small_decoder_graph_matches_eager(side_fold):
    """The captured step equals the eager step token for token, with the ledger
    fold inline and with it on the side stream."""
    from qevict_b200.model import LlamaShape, StickyLlamaDecoder, StickyShape
    shape = LlamaShape(vocab=1000, hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64, ffn=512)
    sticky = StickyShape(omega=16, sink=16, local=32, k_windows=3, q_windows=4, bits=8)
    toks = []
    for mode in ("eager", "graph"):
        m = StickyLlamaDecoder(shape, sticky, batch=2, max_pos=1024, seed=7, std=0.05, side_fold=side_fold)
        ids = torch.randint(0, shape.vocab, (2, 16 + 8 * 16), generator=torch.Generator().manual_seed(1)).cuda()
        m.prefill(ids)
        if mode == "graph":
            m.capture()
        out = []
        for _ in range(40):       # crosses two eviction cycles
            if mode == "graph":
                m.step_graph()
                out.append(m.next_tok.clone())
            else:
                out.append(m.step_eager().clone())
        toks.append(torch.stack(out).cpu())
        assert all(st.read_error() == 0 for st in m.states)
    assert torch.equal(toks[0], toks[1])


@pytest.mark.parametrize("rows,cols", [(1, 128256), (3, 1000)])
def test_argmax(rows, cols):
    g = torch.Generator(device="cuda").manual_seed(cols)
    x = torch.randn(rows, cols, generator=g, device="cuda").to(torch.bfloat16)
    x[0, cols // 3] = 9.0          # a tie between two positions: the smaller index wins
    x[0, cols // 2] = 9.0
    ws = torch.zeros(int(N.lib().qv_argmax_workspace_bytes(rows)), dtype=torch.uint8, device="cuda")
    out = torch.empty(rows, dtype=torch.int64, device="cuda")
    for _ in range(2):             # the workspace is left reusable
        rc = N.lib().qv_argmax(rows, cols, N.ptr(x), N.ptr(out), N.ptr(ws), ws.numel(),
                               torch.cuda.current_stream().cuda_stream)
        N.check(rc, "qv_argmax")
        assert torch.equal(out, torch.argmax(x.float(), dim=1))
        assert int(out[0]) == cols // 3



@pytest.mark.parametrize("rows,n,k", [(1, 4096, 4096), (1, 6144, 4096), (1, 4096, 14336), (3, 1000, 1000),
                                      (8, 257, 2048), (1, 30000, 4096),
                                      # K > 8192: the K-slice layout (ragged slices, several token rows)
                                      (2, 4096, 14336), (3, 1000, 8200), (8, 300, 16384), (1, 7, 9000)])
def test_gemv(rows, n, k):
    """qv_gemv against an fp32 reference: fp32 accumulation, one bf16 rounding."""
    g = torch.Generator(device="cuda").manual_seed(n + k)
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    x = torch.randn(rows, k, generator=g, device="cuda").to(torch.bfloat16)
    y = torch.empty(rows, n, dtype=torch.bfloat16, device="cuda")
    rc = N.lib().qv_gemv(rows, n, k, N.ptr(w), N.ptr(x), N.ptr(y), torch.cuda.current_stream().cuda_stream)
    N.check(rc, "qv_gemv")
    ref = x.double() @ w.double().t()
    # one bf16 rounding (2^-8 relative) plus fp32 summation-order error
    tol = 2.0 ** -8 * ref.abs() + 1e-5 * (x.double().abs() @ w.double().abs().t())
    assert ((y.double() - ref).abs() <= tol).all()
