"""Seeded builds of the reference's own models and engines, shared by the
fixture script (which runs them unpatched on the CPU) and the GPU tests
(which run the same builds with ``asrback_b200.plugin`` installed).

Everything here is test infrastructure over the reference's classes
(``oracle.reference.load()``); nothing is re-implemented.

- :func:`whisper_config1`: BASELINE config 1, the Whisper-tiny architecture
  with nn's default initialisation after ``torch.manual_seed(0)`` and
  log-mel input ``N(0, 1)`` ``[8, 80, 3000]`` drawn from the same continuing
  RNG stream (asrback ``src/asrback/models/whisper.py:73-342``);
- :func:`write_whisper_model_dir`: a checkpoint directory the reference's
  ``Transcriber`` loads (``whisper.py:468-577``): ``config.json``,
  ``model.safetensors``, and a word-level ``tokenizer.json`` whose special
  tokens sit at Whisper's ids, with ``tokenizer_config.json`` naming a few
  language tokens;
- :func:`run_whisper_steps`: the prompt pass and greedy ``Transcriber._step``
  calls (``whisper.py:828-878``, ``:942-960``) on a stub engine, eagerly or
  replayed from the reference's ``CapturedGraph`` (``transcription.py:158-179``);
- :func:`submit_whisper_jobs`: windows queued to a running ``Transcriber``
  and their results (``_Job``, ``_serve``, ``_admit``, ``_advance``,
  ``_finish``: ``whisper.py:728-940``).
"""

from __future__ import annotations

import json
import types
from pathlib import Path

import numpy as np
import torch

SOT, EN, TRANSCRIBE, NO_TIMESTAMPS, EOS = 50258, 50259, 50359, 50363, 50257
WHISPER_PREFIX = [SOT, EN, TRANSCRIBE, NO_TIMESTAMPS]

# Whisper's generation config: token ids never sampled (the multilingual
# checkpoints' list) and the ones suppressed at the first step.
SUPPRESS_TOKENS = [1, 2, 7, 8, 9, 10, 14, 25, 26, 27, 28, 29, 31, 58, 59, 60, 61, 62, 63, 90, 91,
                   92, 93, 359, 503, 522, 542, 873, 893, 902, 918, 922, 931, 1350, 1853, 1982,
                   2460, 2627, 3246, 3253, 3268, 3536, 3846, 3961, 4183, 4667, 6585, 6647, 7273,
                   9061, 9383, 10428, 10929, 11938, 12033, 12331, 12562, 13793, 14157, 14635,
                   15265, 15618, 16553, 16604, 18362, 18956, 20075, 21675, 22520, 26130, 26161,
                   26435, 28279, 29464, 31650, 32302, 32470, 36865, 42863, 47425, 49870, 50254,
                   50258, 50358, 50359, 50360, 50361, 50362]
BEGIN_SUPPRESS = [220, EOS]

WHISPER_TINY = dict(
    d_model=384, encoder_attention_heads=6, decoder_attention_heads=6, encoder_layers=4,
    decoder_layers=4, encoder_ffn_dim=1536, decoder_ffn_dim=1536, num_mel_bins=80,
    max_source_positions=1500, max_target_positions=448, vocab_size=51865,
    eos_token_id=EOS, suppress_tokens=SUPPRESS_TOKENS, begin_suppress_tokens=BEGIN_SUPPRESS)

# Whisper's special tokens after <|endoftext|> (50257): <|startoftranscript|>,
# the language tokens (the first few of 99), then the task and control tokens.
_LANGUAGES = {"en": 50259, "zh": 50260, "de": 50261, "es": 50262, "ru": 50263}
_SPECIAL = {"<|endoftext|>": EOS, "<|startoftranscript|>": SOT, "<|translate|>": 50358,
            "<|transcribe|>": TRANSCRIBE, "<|startoflm|>": 50360, "<|startofprev|>": 50361,
            "<|nospeech|>": 50362, "<|notimestamps|>": NO_TIMESTAMPS}

CONFIG1_STEPS = 64
CONFIG1_BATCH = 8


def whisper_config1(ref) -> tuple[torch.nn.Module, torch.Tensor]:
    """The reference's ``WhisperForConditionalGeneration`` at config 1 (CPU,
    float32, eval mode) and the config's mel batch."""
    torch.manual_seed(0)
    model = ref.whisper.WhisperForConditionalGeneration(dict(WHISPER_TINY))
    mel = torch.randn(CONFIG1_BATCH, WHISPER_TINY["num_mel_bins"], 3000)
    return model.eval(), mel


def suppress_masks(vocab: int) -> tuple[torch.Tensor, torch.Tensor]:
    """The ``Transcriber``'s suppress masks (``whisper.py:536-543``)."""
    suppress = torch.zeros(vocab, dtype=torch.bool)
    suppress[SUPPRESS_TOKENS] = True
    suppress[NO_TIMESTAMPS + 1:] = True
    first = suppress.clone()
    first[BEGIN_SUPPRESS] = True
    return suppress, first


class _RecordingModel:
    """The model as ``_step`` sees it, copying each step's last hidden state
    into ``last`` (a fixed buffer, so the copy is captured in a graph too)."""

    def __init__(self, model, last: torch.Tensor) -> None:
        self._model = model
        self.model = model.model
        self.logits = model.logits
        self.last = last

    def decode(self, *args, **kwargs):
        hidden = self._model.decode(*args, **kwargs)
        self.last.copy_(hidden[:, -1])
        return hidden


def run_whisper_steps(ref, model, mel: torch.Tensor, steps: int, graph: bool,
                      sample_every: int = 4) -> dict:
    """Encoder, ``set_encoder_output``, the 4-token prompt pass with the first
    token chosen as ``_prefill`` does, then ``steps`` greedy
    ``Transcriber._step`` calls over the whole cache (replayed from the
    reference's ``CapturedGraph`` when ``graph``). Returns numpy arrays: a
    sample of the encoder output, the prompt's hidden state, the decode state
    after the steps and the last hidden state every ``sample_every`` steps."""
    whisper = ref.whisper
    device = mel.device
    batch = mel.shape[0]
    config = model.config
    suppress, first_suppress = (m.to(device) for m in suppress_masks(config["vocab_size"]))
    with torch.inference_mode():
        encoded = model.model.encoder(mel)
        cache = model.allocate_cache(batch)
        model.set_encoder_output(cache, encoded)
        tokens = torch.tensor([WHISPER_PREFIX] * batch, device=device)
        positions = torch.arange(config["max_target_positions"], device=device)
        prompt = model.decode(tokens, positions[:4], cache, length=4)
        logits = model.logits(prompt[:, -1]).float()
        stub = types.SimpleNamespace(_suppress=suppress, _eos=EOS)
        stub._choose = types.MethodType(whisper.Transcriber._choose, stub)
        token, logprob = stub._choose(logits, first_suppress, None)
        state = whisper._DecodeState.allocate(batch, config["max_target_positions"], device)
        state.tokens[:, 0] = token
        state.position[:] = 4
        state.end[:] = config["max_target_positions"] - 1
        state.finished[:] = token == EOS
        state.sum_logprobs[:] = logprob
        state.generated[:, 4] = token
        last = torch.zeros((batch, config["d_model"]), dtype=prompt.dtype, device=device)
        stub.model = _RecordingModel(model, last)

        def step():
            whisper.Transcriber._step(stub, state, cache)

        if graph:
            # CapturedGraph warms the step up three times: put the state and
            # the self-attention cache back afterwards (same addresses).
            saved = [t.clone() for t in (state.tokens, state.position, state.finished,
                                         state.sum_logprobs, state.generated,
                                         cache.self_keys, cache.self_values)]
            captured = ref.transcription.CapturedGraph(step)
            for target, value in zip((state.tokens, state.position, state.finished,
                                      state.sum_logprobs, state.generated, cache.self_keys,
                                      cache.self_values), saved):
                target.copy_(value)
            run = captured.replay
        else:
            run = step
        hidden, margins = [], []
        for t in range(steps):
            run()
            if t % sample_every == 0:
                hidden.append(last.float().clone())
            # The top-two margin of the step's logits (suppressed tokens out):
            # a step whose margin is tiny may pick either token.
            top = model.logits(last).float().masked_fill(suppress, -float("inf")).topk(2).values
            margins.append(top[:, 0] - top[:, 1])
        if device.type == "cuda":
            torch.cuda.synchronize(device)
    frames = encoded[:, ::50].float()
    return dict(
        encoder_sample=frames.cpu().numpy(),
        prompt_hidden=prompt[:, -1].float().cpu().numpy(),
        first_token=token.cpu().numpy(),
        generated=state.generated[:, :5 + steps].cpu().numpy(),
        position=state.position.cpu().numpy(),
        finished=state.finished.cpu().numpy(),
        sum_logprobs=state.sum_logprobs.float().cpu().numpy(),
        hidden=torch.stack(hidden, 1).cpu().numpy(),
        margins=torch.stack(margins, 1).cpu().numpy(),
    )


def write_whisper_model_dir(path: Path, model) -> Path:
    """A checkpoint directory for the reference's ``Transcriber``."""
    from safetensors.torch import save_file
    from tokenizers import Tokenizer, models

    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    config = dict(model.config)
    (path / "config.json").write_text(json.dumps(config))
    state = {name: tensor.detach().float().contiguous().cpu()
             for name, tensor in model.state_dict().items()}
    save_file(state, str(path / "model.safetensors"))
    vocab = {f"<t{i}>": i for i in range(config["vocab_size"])}
    names = {**_SPECIAL, **{f"<|{code}|>": index for code, index in _LANGUAGES.items()}}
    for name, index in names.items():
        del vocab[f"<t{index}>"]
        vocab[name] = index
    Tokenizer(models.WordLevel(vocab, unk_token="<t0>")).save(str(path / "tokenizer.json"))
    decoder = {str(index): {"content": name, "special": True} for name, index in names.items()}
    (path / "tokenizer_config.json").write_text(json.dumps({"added_tokens_decoder": decoder}))
    return path


def config1_jobs() -> list[dict]:
    """The eight config-1 windows as engine jobs: two detect their language,
    two carry earlier text (a longer prompt, its own prompt pass)."""
    jobs = []
    for index in range(CONFIG1_BATCH):
        language = None if index in (1, 6) else "en"
        previous = [440 + index, 1029, 7 * index + 300] if index in (3, 5) else []
        jobs.append(dict(language=language, previous=previous))
    return jobs


def submit_whisper_jobs(ref, transcriber, mel: np.ndarray, max_new_tokens: int) -> list[dict]:
    """Queues one ``_Job`` per window to the running ``transcriber`` and waits
    for all results."""
    whisper = ref.whisper
    jobs = []
    for log_mel, spec in zip(mel, config1_jobs()):
        job = whisper._Job(np.asarray(log_mel, dtype=np.float32), spec["previous"],
                           spec["language"], "transcribe", 0.0, max_new_tokens)
        jobs.append(job)
    for job in jobs:
        transcriber._queue.put(job)
    results = [transcriber._worker.wait(job.future) for job in jobs]
    return [dict(language=r.language, tokens=list(r.tokens), avg_logprob=float(r.avg_logprob),
                 no_speech_prob=float(r.no_speech_prob)) for r in results]


# ---------------------------------------------------------------- Qwen3 ----

QWEN3_1_7B_4L = dict(vocab_size=8192, hidden_size=2048, num_hidden_layers=4,
                     num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                     rms_norm_eps=1e-6, intermediate_size=6144)
QWEN3_PROMPTS = [411, 37, 260, 129]
QWEN3_STEPS = 16
QWEN3_BUCKET = 512


def rope_tables(theta: float, head_dim: int, length: int):
    """The reference's RoPE tables (``qwen3_asr.py:795-803``), float32."""
    inverse = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
    angles = torch.arange(length).float()[:, None] * inverse[None, :]
    angles = torch.cat((angles, angles), dim=-1)
    return angles.cos(), angles.sin()


WHISPER_TURBO_4L = dict(
    d_model=1280, encoder_attention_heads=20, decoder_attention_heads=20, encoder_layers=1,
    decoder_layers=4, encoder_ffn_dim=64, decoder_ffn_dim=5120, num_mel_bins=128,
    max_source_positions=1500, max_target_positions=448, vocab_size=51866,
    eos_token_id=EOS)
TURBO_BATCH = 4
TURBO_STEPS = 24


def _seeded_ids(count: int, seed: int, vocab: int) -> torch.Tensor:
    generator = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (count,), generator=generator)


def qwen3_text_model(ref, dtype: torch.dtype, device) -> tuple[torch.nn.Module, torch.nn.Module]:
    """The reference's ``TextModel`` at Qwen3-1.7B widths, 4 layers, and an
    ``lm_head``, with seeded weights (``asrback_b200.synthetic``)."""
    from asrback_b200.synthetic import seeded_parameters

    model = ref.qwen3_asr.TextModel(dict(QWEN3_1_7B_4L))
    lm_head = torch.nn.Linear(QWEN3_1_7B_4L["hidden_size"], QWEN3_1_7B_4L["vocab_size"],
                              bias=False)
    seeded_parameters(model, 3)
    seeded_parameters(lm_head, 4)
    return model.to(device, dtype).eval(), lm_head.to(device, dtype).eval()


def run_qwen3_steps(ref, model, lm_head, forced: torch.Tensor | None, graph: bool) -> dict:
    """Packed causal prefill of four ragged prompts (``TextModel.prefill``,
    ``qwen3_asr.py:463-492``, with ``Segments`` on the padded-SDPA path), then
    ``QWEN3_STEPS`` calls of ``TextModel.step`` (``:494-524``) over the
    ``QWEN3_BUCKET``-position cache view, one token per row at its own
    position; replayed from the reference's ``CapturedGraph`` when ``graph``.
    Step t feeds ``forced[:, t]`` (or, without ``forced``, the previous step's
    argmax). Returns the tokens fed, the argmax and hidden state per step."""
    qwen3 = ref.qwen3_asr
    device = next(model.parameters()).device
    dtype = next(model.parameters()).dtype
    config = QWEN3_1_7B_4L
    batch = len(QWEN3_PROMPTS)
    cos, sin = (t.to(device, dtype) for t in rope_tables(1e6, config["head_dim"], 1024))
    shape = (config["num_hidden_layers"], batch, 1024, config["num_key_value_heads"],
             config["head_dim"])
    cache = qwen3.KVCache(torch.zeros(shape, dtype=dtype, device=device),
                          torch.zeros(shape, dtype=dtype, device=device))
    lengths = list(QWEN3_PROMPTS)
    with torch.inference_mode():
        ids = torch.cat([_seeded_ids(n, 700 + b, config["vocab_size"])
                         for b, n in enumerate(lengths)]).to(device)
        rows = torch.tensor([b for b, n in enumerate(lengths) for _ in range(n)], device=device)
        positions = torch.cat([torch.arange(n) for n in lengths]).to(device)
        segments = qwen3.Segments.from_lengths(lengths, device, False)
        hidden = model.prefill(model.embed_tokens(ids), cache, rows, positions, segments,
                               cos[positions], sin[positions])
        prefill_last = hidden[segments.starts[1:].long() - 1]
        first = lm_head(prefill_last).float().argmax(dim=-1)
        view = cache.narrow(batch, QWEN3_BUCKET)
        tokens = (forced[:, 0].to(device) if forced is not None else first).clone()
        position = torch.tensor(lengths, device=device)
        out = torch.zeros((batch, config["hidden_size"]), dtype=dtype, device=device)

        def step():
            out.copy_(model.step(tokens, position, view, cos, sin, False))

        run = ref.transcription.CapturedGraph(step).replay if graph else step
        fed, argmax, hiddens, top2 = [], [], [], []
        for t in range(QWEN3_STEPS):
            if forced is not None:
                tokens.copy_(forced[:, t])
            fed.append(tokens.clone())
            run()
            logits = lm_head(out).float()
            choice = logits.argmax(dim=-1)
            argmax.append(choice)
            top2.append(logits.topk(2).values)
            hiddens.append(out.float().clone())
            if forced is None:
                tokens.copy_(choice)
            position += 1
    return dict(prefill_last=prefill_last.float().cpu().numpy(),
                first=first.cpu().numpy(),
                tokens=torch.stack(fed, 1).cpu().numpy(),
                argmax=torch.stack(argmax, 1).cpu().numpy(),
                top2=torch.stack(top2, 1).cpu().numpy(),
                hidden=torch.stack(hiddens, 1).cpu().numpy())


def whisper_turbo_decoder(ref, dtype: torch.dtype, device) -> torch.nn.Module:
    """The reference's ``WhisperForConditionalGeneration`` at Whisper
    large-v3-turbo decoder widths (4 layers, 1280 wide, 20 heads) with seeded
    decoder weights; the encoder (one layer, unused here) keeps its default
    initialisation."""
    from asrback_b200.synthetic import seeded_parameters

    torch.manual_seed(1)
    model = ref.whisper.WhisperForConditionalGeneration(dict(WHISPER_TURBO_4L))
    seeded_parameters(model.model.decoder, 1)
    return model.to(device, dtype).eval()


def run_turbo_steps(ref, model, forced: torch.Tensor | None, graph: bool) -> dict:
    """``set_encoder_output`` of ``N(0, 1)`` encoder states, the 4-token
    prompt pass, ``3 * b`` more single-row steps for row b (ragged positions),
    then ``TURBO_STEPS`` fixed-shape steps over the 64-position bucket view
    (``decode(..., length=None)``, ``whisper.py:255-277``), teacher-forced on
    ``forced`` when given; replayed from the reference's ``CapturedGraph``
    when ``graph``."""
    from asrback_b200.synthetic import seeded_normal

    device = next(model.parameters()).device
    dtype = next(model.parameters()).dtype
    batch = TURBO_BATCH
    vocab = model.config["vocab_size"]
    with torch.inference_mode():
        states = seeded_normal((batch, 1500, model.config["d_model"]), 41).to(device, dtype)
        cache = model.allocate_cache(batch)
        model.set_encoder_output(cache, states)
        prefix = torch.tensor([WHISPER_PREFIX] * batch, device=device)
        positions = torch.arange(448, device=device)
        prompt = model.decode(prefix, positions[:4], cache, length=4)
        start = []
        for b in range(batch):
            row = cache.rows(b, b + 1)
            extra = _seeded_ids(3 * b, 800 + b, EOS)
            for i, token in enumerate(extra.tolist()):
                model.decode(torch.tensor([[token]], device=device),
                             torch.tensor([4 + i], device=device), row)
            start.append(4 + 3 * b)
        view = cache.narrow(batch, 64)
        tokens = torch.full((batch, 1), NO_TIMESTAMPS, device=device)
        if forced is not None:
            tokens.copy_(forced[:, :1])
        position = torch.tensor(start, device=device)
        out = torch.zeros((batch, model.config["d_model"]), dtype=dtype, device=device)

        def step():
            out.copy_(model.decode(tokens, position, view)[:, -1])

        run = ref.transcription.CapturedGraph(step).replay if graph else step
        fed, argmax, hiddens, top2 = [], [], [], []
        for t in range(TURBO_STEPS):
            if forced is not None:
                tokens.copy_(forced[:, t:t + 1])
            fed.append(tokens[:, 0].clone())
            run()
            logits = model.logits(out).float()[:, :vocab]
            choice = logits.argmax(dim=-1)
            argmax.append(choice)
            top2.append(logits.topk(2).values)
            hiddens.append(out.float().clone())
            if forced is None:
                tokens.copy_(choice[:, None])
            position += 1
    return dict(prompt_hidden=prompt[:, -1].float().cpu().numpy(),
                tokens=torch.stack(fed, 1).cpu().numpy(),
                argmax=torch.stack(argmax, 1).cpu().numpy(),
                top2=torch.stack(top2, 1).cpu().numpy(),
                hidden=torch.stack(hiddens, 1).cpu().numpy(),
                self_keys=cache.self_keys[:, :, :, :40].float()[:, :, ::5].cpu().numpy())
