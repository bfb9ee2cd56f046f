"""asrback_b200: sm_100a kernels for asrback's attention hot path.

- :mod:`asrback_b200.attention`: the ops (Whisper decode self/cross attention,
  Qwen3 grouped-query decode attention, Whisper encoder attention) over the C
  ABI of ``include/asrback_attn.h``;
- :mod:`asrback_b200.whisper`, :mod:`asrback_b200.qwen3_asr`: the reference's
  modules on the path, running those ops;
- :mod:`asrback_b200.plugin`: patches the reference's own classes in place;
- :mod:`asrback_b200.transcription`: ``CapturedGraph``.
"""

__version__ = "0.1.0"
