"""Drives one implementation of the engine's public API (engine/api/cachepotato.h) through a fixed
conversation and writes what it saw as JSON. Run as a child process (one model per process):

    python tests/chat_driver.py ref|gpu MODEL_PATH OUT_JSON

  ref  oracle/_ref/libcpref_api.so: the reference's own cachepotato.c, engine and tokenizer (CPU)
  gpu  cachepotato_b200/_build/libcachepotato_b200.so (this repository), with the reference's
       tokenizer module (oracle/_ref/libcpref_tok.so) loaded first, as a front-end links it
"""
import ctypes
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

# (message, max_new, stop the turn from the callback after this many tokens or None, reset first)
TURNS = [("Hello there, how are you?", 12, None, False),
         ("Tell me about the weather in 3 words.", 10, None, False),
         ("What is it?", 12, 4, False),
         ("hi", 8, None, True),
         ("And the weather here?", 16, None, False),
         ("Tell me what you are about.", 16, None, False)]
MAX_CTX = 128


class Options(ctypes.Structure):
    _fields_ = [("budget_mb", ctypes.c_long), ("threads", ctypes.c_int), ("pin_cores", ctypes.c_int),
                ("max_ctx", ctypes.c_int), ("tokenizer_dir", ctypes.c_char_p)]


class Turn(ctypes.Structure):
    _fields_ = [("prompt_tokens", ctypes.c_int), ("context_tokens", ctypes.c_int),
                ("generated_tokens", ctypes.c_int), ("context_reset", ctypes.c_int),
                ("prefill_s", ctypes.c_double), ("decode_s", ctypes.c_double), ("stop", ctypes.c_int)]


class Stats(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int), ("d_model", ctypes.c_int), ("n_experts", ctypes.c_int),
                ("topk", ctypes.c_int), ("vocab", ctypes.c_int), ("max_ctx", ctypes.c_int),
                ("threads", ctypes.c_int), ("budget_mb", ctypes.c_long), ("file_bytes", ctypes.c_longlong),
                ("hits", ctypes.c_long), ("misses", ctypes.c_long), ("evictions", ctypes.c_long),
                ("bytes_fetched", ctypes.c_longlong), ("resident_bytes", ctypes.c_longlong)]


TOKEN_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.POINTER(ctypes.c_char), ctypes.c_size_t, ctypes.c_void_p)


def load(kind: str) -> ctypes.CDLL:
    if kind == "ref":
        return ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libcpref_api.so"))
    ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libcpref_tok.so"), mode=ctypes.RTLD_GLOBAL)
    return ctypes.CDLL(os.path.join(ROOT, "cachepotato_b200", "_build", "libcachepotato_b200.so"))


def run(kind: str, model: str) -> dict:
    lib = load(kind)
    lib.cp_open.restype = ctypes.c_void_p
    lib.cp_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(Options), ctypes.c_char_p, ctypes.c_size_t]
    lib.cp_chat.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, TOKEN_FN, ctypes.c_void_p,
                            ctypes.POINTER(Turn)]
    lib.cp_reset.argtypes = [ctypes.c_void_p]
    lib.cp_close.argtypes = [ctypes.c_void_p]
    lib.cp_get_stats.argtypes = [ctypes.c_void_p, ctypes.POINTER(Stats)]
    opt = Options()
    lib.cp_options_default(ctypes.byref(opt))
    opt.budget_mb, opt.threads, opt.max_ctx = -1, 8, MAX_CTX        # CP_BUDGET_NONE
    err = ctypes.create_string_buffer(512)
    m = lib.cp_open(model.encode(), ctypes.byref(opt), err, 512)
    if not m:
        return {"error": err.value.decode()}
    second = lib.cp_open(model.encode(), ctypes.byref(opt), err, 512)      # one model per process
    out = {"second_open_refused": not second, "turns": []}
    for msg, max_new, stop_after, reset in TURNS:
        if reset:
            lib.cp_reset(m)
        got = []

        def on_token(p, n, user, got=got, stop_after=stop_after):
            got.append(ctypes.string_at(p, n).hex())
            return 1 if stop_after is not None and len(got) >= stop_after else 0

        fn = TOKEN_FN(on_token)
        t = Turn()
        rc = lib.cp_chat(m, msg.encode(), max_new, fn, None, ctypes.byref(t))
        out["turns"].append({"rc": rc, "tokens": got, "prompt_tokens": t.prompt_tokens,
                             "context_tokens": t.context_tokens, "generated_tokens": t.generated_tokens,
                             "context_reset": t.context_reset, "stop": t.stop})
    st = Stats()
    lib.cp_get_stats(m, ctypes.byref(st))
    out["stats"] = {k: getattr(st, k) for k in ("n_layers", "d_model", "n_experts", "topk", "vocab", "max_ctx")}
    lib.cp_close(m)
    return out


if __name__ == "__main__":
    kind, model, path = sys.argv[1:4]
    res = run(kind, model)
    with open(path, "w") as f:
        json.dump(res, f)
