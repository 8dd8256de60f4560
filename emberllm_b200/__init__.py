"""emberllm_b200 — emberllm's token loop (decode + prefill of Q8_0/Q4_0 LLaMA-family
decoders) on NVIDIA B200, behind emberllm's own C API.

The product is the C-ABI library ``libember_b200.so`` (C11 host code + sm_100a
CUDA kernels, built by ``make -C emberllm_b200``). This package is its Python
face and mirrors emberllm's ctypes ``Ember`` class
(bindings/python/emberllm.py:112-201) for the parts on the token loop: load a
model, create a run state, prefill, forward, and greedy generation over token
ids. Text tokenization stays with emberllm's tokenizer (host code outside the
token loop), so this mirror works on ids.
"""
import ctypes

from . import _lib as _libmod
from ._lib import EmberHeader, cuda_available, load

__all__ = ["Ember", "EmberBatch", "Sampler", "EmberHeader", "cuda_available", "load"]


class Ember:
    """A loaded model and one run state (mirrors emberllm's Python ``Ember``)."""

    def __init__(self, path, ctx=0, kv_fp16=False):
        self.lib = load()
        self.m = self.lib.ember_model_load(str(path).encode())
        if not self.m:
            raise RuntimeError(f"failed to load model: {path}")
        self.header = self.lib.ember_model_header(self.m).contents
        self.st = self.lib.ember_state_new_ex(self.m, int(ctx), 1 if kv_fp16 else 0)
        maxs = self.header.max_seq_len
        self.ctx = maxs if ctx <= 0 or ctx > maxs else ctx
        self.vocab = self.header.vocab_size

    # -- token loop --------------------------------------------------------
    def forward(self, tok, pos):
        """Logits (a ctypes float array view of vocab_size) after token ``tok`` at ``pos``."""
        return self.lib.ember_forward(self.m, self.st, int(tok), int(pos))

    def prefill(self, ids, start=0):
        arr = (ctypes.c_int * len(ids))(*ids)
        return self.lib.ember_prefill(self.m, self.st, arr, len(ids), int(start))

    def logits_list(self, ptr):
        return [ptr[i] for i in range(self.vocab)]

    def greedy(self, first_tok, pos, n):
        """n greedy steps on the device; returns the n chosen token ids."""
        out = (ctypes.c_int * n)()
        self.lib.ember_forward_greedy(self.m, self.st, int(first_tok), int(pos), int(n), out)
        return list(out)

    def generate_ids(self, prompt_ids, max_tokens=128):
        """Greedy continuation of ``prompt_ids`` (ids in, ids out), as the
        reference's generate loop with temperature 0 (ref src/main.c:189-206)."""
        logits = self.prefill(prompt_ids)
        best = max(range(self.vocab), key=lambda i: (logits[i], -i))
        if max_tokens <= 1:
            return [best][:max_tokens]
        return [best] + self.greedy(best, len(prompt_ids), max_tokens - 1)

    def sample(self, sampler):
        """Draw the next token from the logits of the last forward / prefill on
        the device with ``sampler``'s settings, random stream and history, then
        record it in the history, as the reference's ember_sample does
        (src/sample.c:120-175)."""
        return sampler.sample_device(self)

    # -- lifetime ----------------------------------------------------------
    def close(self):
        if getattr(self, "st", None):
            self.lib.ember_state_free(self.st)
            self.st = None
        if getattr(self, "m", None):
            self.lib.ember_model_free(self.m)
            self.m = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        self.close()


class EmberBatch:
    """Independent sequences decoded together on one model (the library's
    ember_batch_* extension): per-stream prompts, then greedy steps of all
    streams at once. Each stream's tokens equal its own single-sequence run."""

    def __init__(self, ember, n_streams, ctx=0, kv_fp16=False, max_steps=256):
        self.lib = ember.lib
        self.vocab = ember.vocab
        self.n = int(n_streams)
        self.b = self.lib.ember_batch_new(ember.m, self.n, int(ctx), 1 if kv_fp16 else 0, int(max_steps))

    def prefill(self, stream, ids):
        """Prompt of one stream; returns the index of its greedy next token."""
        arr = (ctypes.c_int * len(ids))(*[int(i) for i in ids])
        p = self.lib.ember_batch_prefill(self.b, int(stream), arr, len(ids))
        best, bv = 0, p[0]
        for i in range(1, self.vocab):
            if p[i] > bv:
                best, bv = i, p[i]
        return best

    def greedy(self, toks, pos, n_steps, logits=False):
        """n_steps greedy steps of every stream; returns tokens [n_steps][n] (and
        the last step's logits [n][vocab] when asked)."""
        t = (ctypes.c_int * self.n)(*[int(x) for x in toks])
        p = (ctypes.c_int * self.n)(*[int(x) for x in pos])
        out = (ctypes.c_int * (n_steps * self.n))()
        lg = (ctypes.c_float * (self.n * self.vocab))() if logits else None
        self.lib.ember_batch_greedy(self.b, t, p, int(n_steps), out,
                                    ctypes.cast(lg, ctypes.POINTER(ctypes.c_float)) if logits else None)
        toks_out = [[out[s * self.n + i] for i in range(self.n)] for s in range(n_steps)]
        return (toks_out, lg) if logits else toks_out

    def close(self):
        if getattr(self, "b", None):
            self.lib.ember_batch_free(self.b)
            self.b = None



class Sampler:
    """The reference's EmberSampler (src/ember.h:141-155, src/sample.c:17-67) on
    the host: settings, the xorshift64* state and the ring of recent tokens.
    Drawing runs on the device (``Ember.sample``); the history ring and the
    random stream advance exactly as the reference's."""

    def __init__(self, temperature=0.0, top_p=1.0, top_k=0, seed=0):
        self.temperature, self.top_p, self.top_k = float(temperature), float(top_p), int(top_k)
        self.min_p, self.repeat_penalty = 0.0, 1.0
        self.presence_penalty = self.frequency_penalty = 0.0
        self.repeat_last_n = 0
        self.rng_state = ctypes.c_uint64(seed if seed else 0x9E3779B97F4A7C15)
        self.history = None
        self.hist_len = self.hist_pos = 0

    def set_penalties(self, repeat_penalty=1.0, repeat_last_n=0, presence_penalty=0.0, frequency_penalty=0.0,
                      min_p=0.0):
        """as ember_sampler_set_penalties: a history of repeat_last_n tokens only
        when some penalty is active; the history restarts empty"""
        self.repeat_penalty, self.repeat_last_n = float(repeat_penalty), int(repeat_last_n)
        self.presence_penalty, self.frequency_penalty = float(presence_penalty), float(frequency_penalty)
        self.min_p = float(min_p)
        need = self.repeat_last_n > 0 and (self.repeat_penalty != 1.0 or self.presence_penalty != 0.0
                                           or self.frequency_penalty != 0.0)
        self.history = (ctypes.c_int * self.repeat_last_n)() if need else None
        self.hist_len = self.hist_pos = 0

    def accept(self, token):
        """record an emitted token in the ring (ember_sampler_accept)"""
        if self.history is None:
            return
        self.history[self.hist_pos] = int(token)
        self.hist_pos = (self.hist_pos + 1) % len(self.history)
        if self.hist_len < len(self.history):
            self.hist_len += 1

    def reset(self):
        self.hist_len = self.hist_pos = 0

    def params(self):
        return _libmod.EmberSampleParams(self.temperature, self.top_p, self.top_k, self.min_p,
                                         self.repeat_penalty, self.presence_penalty, self.frequency_penalty)

    def sample_device(self, ember):
        p = self.params()
        tok = ember.lib.ember_sample_device(ember.st, ctypes.byref(p), ctypes.byref(self.rng_state),
                                            self.history if self.hist_len else None, self.hist_len)
        self.accept(tok)
        return tok
