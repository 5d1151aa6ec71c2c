"""The tensor-core output projection (tcgen05 + TMA) and the projection ->
sampler launch pair.

The projection is checked against a float64 product of the same bf16 inputs:
each logit must lie within half a bf16 ulp plus the fp32 accumulation bound of
the exact value, and against torch's bf16 matmul (the reference's nn.Linear on
cuBLAS) it may differ only by one bf16 ulp, rarely.  The sampler that follows
is compared bit for bit with the CPU oracle run on the very logits the
projection wrote."""

import numpy as np
import pytest
import torch

from mapperatorinator_b200 import _native as N
from mapperatorinator_b200 import sampling as S
from oracle import oracle
from tests.harness import workloads as W
from tests.harness.stepargs import DeviceStep

pytestmark = pytest.mark.gpu


def _inputs(device, rows, d, vocab, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    h = torch.randn((rows, d), generator=g, device=device).to(torch.bfloat16)
    w = (torch.randn((vocab, d), generator=g, device=device) * 0.02).to(torch.bfloat16)
    return h, w


def _bf16_ulp(x: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 numbers at |x| (8 significant bits)."""
    ax = x.abs().clamp_min(2.0 ** -126)
    return torch.exp2(torch.floor(torch.log2(ax)) - 7)


@pytest.mark.parametrize("rows,d,vocab,tile_n", [
    (256, 768, 4096, 0), (256, 768, 4096, 64), (256, 768, 4096, 128),  # the config-3 projection
    (130, 128, 520, 0),    # ragged rows and vocabulary (partial tiles on both axes)
    (1, 64, 64, 64),       # one row, one k-block
    (384, 1024, 8192, 128),
])
def test_projection_within_float64_bound(cuda_device, rows, d, vocab, tile_n):
    h, w = _inputs(cuda_device, rows, d, vocab, seed=rows * 7 + d + vocab)
    out = S.lm_head_logits(h, w, tile_n=tile_n)
    torch.cuda.synchronize()
    exact = h.double() @ w.double().T
    absdot = h.double().abs() @ w.double().abs().T
    # fp32 accumulation of d products (each exact in fp32): |err| <= d * 2^-24 * sum |h w|
    bound = 0.5 * _bf16_ulp(exact) * (1 + 2.0 ** -7) + d * 2.0 ** -24 * absdot
    err = (out.double() - exact).abs()
    assert bool((err <= bound).all()), float((err - bound).max())
    # nearly every logit is the correctly rounded bf16 of the exact value
    rn = exact.float().to(torch.bfloat16)  # exact is within 2^-24 relative of its fp32 rounding
    assert float((out == rn).double().mean()) > 0.995


def test_projection_against_cublas(cuda_device):
    # cuBLAS (the reference's proj_out) and the tcgen05 kernel accumulate in
    # different orders: both meet the same float64 bound, so they differ by at
    # most twice it, and they agree on almost every logit
    h, w = _inputs(cuda_device, 256, 768, 4096, seed=5)
    out = S.lm_head_logits(h, w)
    ref = h @ w.T
    torch.cuda.synchronize()
    exact = h.double() @ w.double().T
    bound = 0.5 * _bf16_ulp(exact) * (1 + 2.0 ** -7) + 768 * 2.0 ** -24 * (h.double().abs() @ w.double().abs().T)
    assert bool(((ref.double() - exact).abs() <= bound).all())
    assert bool(((out.double() - ref.double()).abs() <= 2 * bound).all())
    assert float((out != ref).double().mean()) < 0.01


def test_projection_then_sampler_matches_oracle(cuda_device):
    # config 3: 256 hidden rows = 128 CFG pairs x d=768 -> V=4096 bf16 logits ->
    # the config-1 chain (CFG, monotonic state, grammar, temperature on time
    # shifts, top_p 0.9, draw); the sampler is a programmatic dependent launch
    pairs, d, V = 128, 768, 4096
    s = W.batched_decode(seed=33, pairs=pairs, vocab=V).with_(want_scores=True, want_logprobs=True)
    h, w = _inputs(cuda_device, 2 * pairs, d, V, seed=34)
    logits = torch.empty((2 * pairs, V), dtype=torch.bfloat16, device=cuda_device)
    dev = DeviceStep(s, cuda_device)
    dev.args.logits = logits.data_ptr()
    lm = N.new_lmhead_args()
    lm.hidden, lm.hidden_row_stride = h.data_ptr(), h.stride(0)
    lm.weight, lm.weight_row_stride = w.data_ptr(), w.stride(0)
    lm.logits, lm.logits_row_stride = logits.data_ptr(), logits.stride(0)
    lm.rows, lm.d_model, lm.vocab = 2 * pairs, d, V
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    lm.error_word = err.data_ptr()
    N.lmhead_sample_launch(lm, dev.args, torch.cuda.current_stream(cuda_device).cuda_stream)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = dev.results()
    host = s.with_(logits=logits.view(torch.int16).cpu().numpy().view(np.uint16))
    ref = oracle.run(host)
    errs = oracle.compare(ref, got)
    assert not errs, "\n".join(errs)
    # the projection inside the pair wrote what the projection alone writes
    assert torch.equal(logits, S.lm_head_logits(h, w))


def test_fused_sampler_step_hidden(cuda_device):
    pairs, d, V = 64, 768, 4096
    h, w = _inputs(cuda_device, 2 * pairs, d, V, seed=35)
    u = torch.rand(pairs, device=cuda_device)

    def make():
        return S.FusedSampler(vocab_size=V, num_rows=pairs, device=cuda_device, cfg_scale=1.5,
                              time_shift_range=(0, 2000), temperature=0.9, top_p=0.9)

    a, b = make(), make()
    ids_a = a.step_hidden(h, w, uniforms=u).clone()
    ids_b = b.step(S.lm_head_logits(h, w), uniforms=u).clone()
    torch.cuda.synchronize()
    assert torch.equal(ids_a, ids_b)
    assert torch.equal(a.mono_state, b.mono_state)
    with pytest.raises(ValueError):
        a.step_hidden(h[:10], w, uniforms=u)
