"""Greedy step epilogue on the GPU: asrback_greedy_step (through the C ABI)
against the reference's recorded ``_step`` results, the CPU oracle, and at
full size the reference's own GPU expression (``(weight @ rows.T).T.float()``,
``masked_fill``, ``argmax``, ``log_softmax``) on the same tensors.

Tokens must be identical except on rows whose two largest logits lie within
one bf16 rounding step (there the fp32 sums of two summation orders may round
apart). Log-probabilities: max-abs 1e-4; full size, against cuBLAS: 1e-3.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from asrback_b200 import _native, attention, step
from oracle import step as oracle_step
from tests.golden import load
from tests.step_fixtures import initial_state, step_weight

pytestmark = pytest.mark.gpu

DEV = "cuda"
DTYPES = {"fp32": torch.float32, "bf16": torch.bfloat16}


@pytest.fixture(autouse=True)
def clean_status():
    attention.read_status()
    yield


def _near_tie(logits: np.ndarray, bf16: bool) -> np.ndarray:
    """Rows whose two largest (masked) logits are within one rounding step."""
    top = np.sort(logits, axis=1)[:, -2:]
    step_ = np.abs(top[:, 1]) * (2.0 ** -7 if bf16 else 1e-5) + 1e-6
    return top[:, 1] - top[:, 0] <= step_


def _device_state(host: dict, family: str) -> dict:
    tokens = torch.from_numpy(host["tokens"]).to(DEV)
    if family == "whisper":
        tokens = tokens[:, None].contiguous()  # (batch, 1), as the reference keeps it
    return dict(tokens=tokens,
                position=torch.from_numpy(host["position"]).to(DEV),
                end=torch.from_numpy(host["end"]).to(DEV),
                finished=torch.from_numpy(host["finished"]).to(DEV),
                sum_logprobs=torch.from_numpy(host["sum_logprobs"]).to(DEV),
                generated=torch.from_numpy(host["generated"]).to(DEV))


def _check_state(dev: dict, host: dict) -> None:
    for name in ("position", "finished", "generated"):
        np.testing.assert_array_equal(dev[name].cpu().numpy(), host[name], err_msg=name)
    np.testing.assert_array_equal(dev["tokens"].reshape(-1).cpu().numpy(), host["tokens"])
    np.testing.assert_allclose(dev["sum_logprobs"].cpu().numpy(), host["sum_logprobs"],
                               atol=1e-4, rtol=0)


@pytest.mark.parametrize("tag", ["fp32", "bf16"])
@pytest.mark.parametrize("family", ["whisper", "qwen3"])
def test_step_matches_reference(family, tag):
    dtype = DTYPES[tag]
    bf16 = tag == "bf16"
    g = load(f"step_epilogue_{tag}")
    info = g["meta"][family]
    weight = step_weight(family, g["meta"], bf16).to(DEV)
    weight_np = weight.float().cpu().numpy()
    suppress_np = g.get(f"{family}_suppress")
    suppress = None if suppress_np is None else torch.from_numpy(suppress_np).to(DEV)
    host = initial_state(g, family)
    dev = _device_state(host, family)
    exact = True
    for i in range(g["meta"]["steps"]):
        hidden = torch.from_numpy(g[f"{family}_hidden"][i]).to(DEV, dtype)
        token, logprob = step.greedy_choose(hidden, weight, suppress)
        token, logprob = token.cpu().numpy(), logprob.cpu().numpy()
        logits = oracle_step.logits(weight_np, g[f"{family}_hidden"][i], bf16)
        if suppress_np is not None:
            logits[:, suppress_np] = -np.inf
        want = g[f"{family}_token"][i]
        differ = token != want
        assert not (differ & ~_near_tie(logits, bf16)).any(), (token, want)
        exact &= not differ.any()
        np.testing.assert_allclose(logprob[~differ], g[f"{family}_logprob"][i][~differ],
                                   atol=1e-4, rtol=0)
        step.greedy_step(hidden, weight, dev["tokens"], dev["position"], dev["end"],
                         dev["finished"], dev["sum_logprobs"], dev["generated"], info["eos"],
                         suppress)
        host = oracle_step.update_state(host, token, logprob, info["eos"])
        _check_state(dev, host)
    if exact:  # the reference's own state after its steps
        np.testing.assert_array_equal(dev["generated"].cpu().numpy(), g[f"{family}_generated"])
        np.testing.assert_array_equal(dev["finished"].cpu().numpy(),
                                      g[f"{family}_after_finished"][-1])
    assert attention.read_status() == 0


@pytest.mark.parametrize("vocab,width,batch", [
    (51866, 1280, 64),    # Whisper large-v3-turbo, the headline widths
    (151936, 2048, 64),   # Qwen3-ASR-1.7B lm_head, config 4
    (151936, 1024, 64),   # Qwen3-0.6B, config 5
    (51866, 1280, 1),
    (50000, 512, 128),    # the 128-row tile
    (1000, 1000, 100),    # ragged vocabulary tile, width not a multiple of 64
])
def test_full_size_matches_torch(vocab, width, batch):
    gen = torch.Generator(device=DEV).manual_seed(vocab + width + batch)
    weight = (torch.randn((vocab, width), generator=gen, device=DEV) * 0.02).to(torch.bfloat16)
    hidden = torch.randn((batch, width), generator=gen, device=DEV).to(torch.bfloat16)
    suppress = torch.rand(vocab, generator=gen, device=DEV) < 0.05
    token, logprob = step.greedy_choose(hidden, weight, suppress)
    logits = (weight @ hidden.T).T.float().masked_fill(suppress, -float("inf"))
    want = logits.argmax(dim=-1)
    want_lp = torch.log_softmax(logits, dim=-1).gather(1, want[:, None])[:, 0]
    agree = token == want
    assert agree.float().mean().item() >= 0.99
    # Where they differ, ours is a maximum of torch's logits up to one bf16 step.
    top = logits.gather(1, want[:, None])[:, 0]
    ours = logits.gather(1, token[:, None])[:, 0]
    assert torch.all(ours >= top - top.abs() * 2.0 ** -7 - 1e-6)
    torch.testing.assert_close(logprob[agree], want_lp[agree], atol=1e-3, rtol=0)
    assert attention.read_status() == 0


def test_graph_replays_advance_the_state():
    """Captured once, replayed five times: every replay finds the ticket
    counter at zero and advances the state as five oracle steps do."""
    from asrback_b200.transcription import CapturedGraph

    gen = torch.Generator(device=DEV).manual_seed(9)
    vocab, width, batch, length = 3000, 256, 16, 32
    weight = (torch.randn((vocab, width), generator=gen, device=DEV) * 0.05).to(torch.bfloat16)
    hidden = torch.randn((batch, width), generator=gen, device=DEV).to(torch.bfloat16)
    host = dict(tokens=np.arange(batch, dtype=np.int64), position=np.arange(batch) % 4,
                end=np.full(batch, 30, np.int64), finished=np.arange(batch) % 5 == 4,
                sum_logprobs=np.zeros(batch, np.float32),
                generated=np.zeros((batch, length), np.int64))
    host["position"] = host["position"].astype(np.int64)
    dev = _device_state(host, "qwen3")
    eos = [int(torch.argmax((weight.float() @ hidden.float().T)[:, 3]).item())]

    def run():
        step.greedy_step(hidden, weight, dev["tokens"], dev["position"], dev["end"],
                         dev["finished"], dev["sum_logprobs"], dev["generated"], eos)

    run()  # warm-up: allocates the workspace
    host = oracle_step.greedy_step(weight.float().cpu().numpy(), hidden.float().cpu().numpy(),
                                   host, eos, bf16=True)[2]
    graph = CapturedGraph(run)
    # CapturedGraph's warm-up ran the step three more times.
    for _ in range(3 + 5):
        if _ >= 3:
            graph.replay()
        host = oracle_step.greedy_step(weight.float().cpu().numpy(), hidden.float().cpu().numpy(),
                                       host, eos, bf16=True)[2]
    torch.cuda.synchronize()
    _check_state(dev, host)
    assert host["finished"][3]  # row 3 chose EOS


def test_position_past_generated_is_flagged():
    vocab, width, batch = 512, 64, 2
    weight = torch.randn((vocab, width), device=DEV).to(torch.bfloat16)
    hidden = torch.randn((batch, width), device=DEV).to(torch.bfloat16)
    tokens = torch.zeros(batch, dtype=torch.int64, device=DEV)
    position = torch.tensor([3, 7], dtype=torch.int64, device=DEV)  # row 1 advances to 8
    end = torch.full((batch,), 100, dtype=torch.int64, device=DEV)
    finished = torch.zeros(batch, dtype=torch.bool, device=DEV)
    sums = torch.zeros(batch, device=DEV)
    generated = torch.zeros((batch, 8), dtype=torch.int64, device=DEV)
    step.greedy_step(hidden, weight, tokens, position, end, finished, sums, generated, [1])
    torch.cuda.synchronize()
    assert attention.read_status() & _native.STATUS_POSITION
    assert generated[1].eq(0).all() and generated[0, 4] == tokens[0]


def test_suppress_leaves_one_token():
    vocab, width = 4096, 128
    weight = torch.randn((vocab, width), device=DEV).to(torch.bfloat16)
    hidden = torch.randn((3, width), device=DEV).to(torch.bfloat16)
    suppress = torch.ones(vocab, dtype=torch.bool, device=DEV)
    suppress[1234] = False
    token, logprob = step.greedy_choose(hidden, weight, suppress)
    assert token.tolist() == [1234] * 3
    assert torch.all(logprob == 0)
