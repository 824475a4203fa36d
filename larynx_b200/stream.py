"""Chunked (streaming) token -> mel on the B200 Flow decoder.

The driver mirrors CosyVoice3's streaming token2wav loop around the
reference's flow inference (flow_reference.py:531-563): speech tokens arrive
in chunks; whenever `hop` new tokens plus the PreLookahead look-ahead (3
tokens) are available, the flow runs over the prompt and every token so far
with finalize=False (the last 3 tokens are look-ahead context) and the mel
frames of the `hop` new tokens are emitted; `finish()` runs finalize=True
over all tokens and emits the rest.  Every call recomputes the whole
sequence (no cross-call state on the device), with the CFM noise sliced from
frame 0 of the same bank each time, so a frame's noise never changes between
calls.  Frames already emitted are not revised: a later call recomputes them
with more look-ahead and can differ slightly, as in the reference's streaming
use.

`chunk` > 0 runs the estimator with the block-causal chunk mask (upstream
CosyVoice3's streaming attention, static_chunk_size frames); 0 keeps the
reference restatement's full attention.
"""

from __future__ import annotations

from typing import List, Optional, Sequence

import numpy as np

from .flow import PRE_LOOKAHEAD, FlowDecoder, FlowError

TOKEN_MEL_RATIO = 2


class FlowStreamer:
    def __init__(self, decoder: FlowDecoder, prompt_tokens: Sequence[int], prompt_feat, spk_embedding,
                 noise_z=None, hop: int = 25, chunk: int = 0):
        if hop <= 0:
            raise ValueError("hop must be positive")
        self.dec = decoder
        self.prompt_tokens = np.asarray(prompt_tokens, np.int32).reshape(-1)
        self.prompt_feat = np.asarray(prompt_feat, np.float32).reshape(-1, 80)
        self.spk = np.asarray(spk_embedding, np.float32).reshape(-1)
        self.noise_z = None if noise_z is None else np.asarray(noise_z, np.float32).reshape(80, -1)
        self.hop = int(hop)
        self.chunk = int(chunk)
        self.tokens: List[int] = []
        self.emitted_tokens = 0   # tokens whose mel frames have been emitted
        self.finished = False
        self.calls = 0

    def _run(self, n_tokens: int, finalize: bool) -> np.ndarray:
        mel = self.dec.infer(self.prompt_tokens, self.tokens[:n_tokens], self.prompt_feat, self.spk,
                             noise_z=self.noise_z, finalize=finalize, chunk=self.chunk)
        if mel is None:
            raise FlowError(f"flow inference failed: {self.dec.last_error}")
        self.calls += 1
        return mel

    def push(self, tokens: Sequence[int]) -> np.ndarray:
        """Append tokens; returns the newly final mel frames [80, k] (k may be 0)."""
        if self.finished:
            raise FlowError("push after finish")
        self.tokens.extend(int(t) for t in np.asarray(tokens).reshape(-1))
        out = []
        while len(self.tokens) - self.emitted_tokens >= self.hop + PRE_LOOKAHEAD:
            upto = self.emitted_tokens + self.hop
            mel = self._run(upto + PRE_LOOKAHEAD, finalize=False)   # frames of tokens [0, upto) after the prompt
            out.append(mel[:, TOKEN_MEL_RATIO * self.emitted_tokens: TOKEN_MEL_RATIO * upto])
            self.emitted_tokens = upto
        return np.concatenate(out, axis=1) if out else np.zeros((80, 0), np.float32)

    def finish(self) -> np.ndarray:
        """Run the final (finalize=True) call; returns the remaining frames."""
        if self.finished:
            return np.zeros((80, 0), np.float32)
        self.finished = True
        if not self.tokens:
            return np.zeros((80, 0), np.float32)
        mel = self._run(len(self.tokens), finalize=True)
        return mel[:, TOKEN_MEL_RATIO * self.emitted_tokens:]
