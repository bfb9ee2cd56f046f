"""asrback_b200: sm_100a kernels for asrback's attention hot path.

- :mod:`asrback_b200.attention`: the ops (Whisper decode self/cross attention
  and the prompt pass, Qwen3 grouped-query decode attention, Whisper encoder
  attention, varlen attention within packed segments, the cross-attention
  key/value projection) over the C ABI of ``include/asrback_attn.h``;
- :mod:`asrback_b200.step`: the greedy step epilogue (logits, ``_choose``,
  the decode-state update) in one launch;
- :mod:`asrback_b200.plugin`: patches the reference's own classes in place, so
  its models, engine and graph capture run these ops;
- :mod:`asrback_b200.transcription`: ``CapturedGraph``;
- :mod:`asrback_b200.replicas`: one replica per GPU (dispatch, timing).
"""

__version__ = "0.2.0"
