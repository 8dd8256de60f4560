"""ctypes access to the reference's sampler (EmberSampler, ref src/ember.h:141-155)
and to the oracle's restatement of it, for the sampling tests."""
import ctypes

import numpy as np

from . import helpers as H


class RefSampler(ctypes.Structure):
    """Layout of the reference's EmberSampler (ref src/ember.h:141-155)."""
    _fields_ = [("temperature", ctypes.c_float), ("top_p", ctypes.c_float), ("top_k", ctypes.c_int),
                ("min_p", ctypes.c_float), ("repeat_penalty", ctypes.c_float),
                ("presence_penalty", ctypes.c_float), ("frequency_penalty", ctypes.c_float),
                ("repeat_last_n", ctypes.c_int), ("rng_state", ctypes.c_uint64),
                ("history", ctypes.POINTER(ctypes.c_int)), ("hist_cap", ctypes.c_int),
                ("hist_len", ctypes.c_int), ("hist_pos", ctypes.c_int)]


# (temperature, top_p, top_k, min_p, repeat_penalty, repeat_last_n, presence, frequency)
SETTINGS = [
    (0.0, 1.0, 0, 0.0, 1.0, 0, 0.0, 0.0),          # greedy
    (0.8, 0.9, 40, 0.0, 1.0, 0, 0.0, 0.0),         # the CLI's defaults
    (1.0, 1.0, 0, 0.0, 1.0, 0, 0.0, 0.0),          # the whole vocabulary
    (1.3, 0.95, 0, 0.0, 1.0, 0, 0.0, 0.0),         # nucleus only
    (0.7, 1.0, 0, 0.05, 1.0, 0, 0.0, 0.0),         # min-p only
    (0.9, 0.8, 100, 0.02, 1.1, 16, 0.5, 0.3),      # everything, with penalties
    (0.0, 1.0, 0, 0.0, 1.3, 8, 0.2, 0.1),          # greedy after penalties
]


def ref_lib():
    lib = ctypes.CDLL(H.REF_DET)
    lib.ember_sampler_init.argtypes = [ctypes.POINTER(RefSampler), ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                       ctypes.c_uint64]
    lib.ember_sampler_set_penalties.argtypes = [ctypes.POINTER(RefSampler), ctypes.c_float, ctypes.c_int,
                                                ctypes.c_float, ctypes.c_float, ctypes.c_float]
    lib.ember_sample.restype = ctypes.c_int
    lib.ember_sample.argtypes = [ctypes.POINTER(RefSampler), ctypes.POINTER(ctypes.c_float), ctypes.c_int]
    lib.ember_sampler_accept.argtypes = [ctypes.POINTER(RefSampler), ctypes.c_int]
    lib.ember_sampler_free.argtypes = [ctypes.POINTER(RefSampler)]
    lib.ember_sampler_reset.argtypes = [ctypes.POINTER(RefSampler)]
    return lib


def new_ref_sampler(lib, setting, seed):
    temp, top_p, top_k, min_p, rp, last_n, pres, freq = setting
    s = RefSampler()
    lib.ember_sampler_init(ctypes.byref(s), temp, top_p, top_k, seed)
    lib.ember_sampler_set_penalties(ctypes.byref(s), rp, last_n, pres, freq, min_p)
    return s


def history_of(s):
    """the sampler's history array and length as the reference scans them"""
    if not s.history or s.hist_len == 0:
        return None, 0
    return np.ctypeslib.as_array(s.history, (s.hist_cap,)).astype(np.int32).copy(), int(s.hist_len)


def oracle_sample(orc, logits, setting, rng, hist, hist_len):
    """the oracle's sampler on a copy of the logits; returns (token, new rng)"""
    lib = orc.lib
    lib.orc_sample.restype = ctypes.c_int
    lib.orc_sample.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_int] + [ctypes.c_float] * 2 + \
        [ctypes.c_int] + [ctypes.c_float] * 4 + [ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_int),
                                                 ctypes.c_int]
    temp, top_p, top_k, min_p, rp, last_n, pres, freq = setting
    lg = np.ascontiguousarray(logits, np.float32).copy()
    st = ctypes.c_uint64(rng)
    hp = hist.ctypes.data_as(ctypes.POINTER(ctypes.c_int)) if hist is not None else None
    tok = lib.orc_sample(lg.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), len(lg), temp, top_p, top_k, min_p,
                         rp, pres, freq, ctypes.byref(st), hp, hist_len)
    return tok, st.value
