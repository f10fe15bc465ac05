"""The device sampler (temperature, top-k, top-p) against upstream's own
q_sample_token (src/main.c:852-991), compiled from the upstream sources into
oracle/_ref, on the same logits with the same xorshift64* stream.

Both libraries keep one random state per host thread, seeded 123456789, so
each comparison runs in a fresh thread where both streams start together.
Probabilities are formed in a different summation order than upstream's, so
a draw that lands within a few ulps of a bucket boundary could differ; over
the sizes here that chance is negligible and the token sequences must match.
Upstream's sampler reads an unset keep-mask when neither top-k nor top-p is
on (malloc'd memory), so that setting is compared only for validity.
Upstream sorts with a recursive quicksort whose depth grows with the number
of equal probabilities, and its polynomial exp makes every token more than
about 2.2 (after the temperature) below the maximum exactly 0; over a
128256-token vocabulary that recursion overflows a thread's stack.  The
large-vocabulary cases therefore use logits within a few units of each
other (every probability non-zero), and the reference runs on a thread with
a large stack.
"""
import ctypes as C
import threading

import numpy as np
import pytest

import oracle as O
import qorus_b200 as Q

pytestmark = pytest.mark.gpu

needs_ref = pytest.mark.skipif(O.ref is None, reason="oracle/_ref (upstream build) not present")


def in_fresh_thread(fn):
    threading.stack_size(512 << 20)
    box = {}

    def run():
        try:
            box["v"] = fn()
        except BaseException as e:  # noqa: BLE001
            box["e"] = e
    t = threading.Thread(target=run)
    t.start()
    t.join()
    threading.stack_size(0)
    if "e" in box:
        raise box["e"]
    return box["v"]


def draws(lib, logits, temp, k, p, n):
    out = C.c_uint32()
    toks = []
    for _ in range(n):
        rc = lib.q_sample_token(C.c_void_p(logits.ctypes.data), C.c_uint32(logits.size), C.c_float(temp),
                                C.c_uint32(k), C.c_float(p), C.byref(out), None)
        assert rc == 0
        toks.append(out.value)
    return toks


@needs_ref
@pytest.mark.parametrize("temp,k,p", [(0.8, 40, 0.0), (1.0, 0, 0.9), (1.3, 1000, 0.5), (0.5, 5, 0.95),
                                      (2.0, 0, 0.3), (1.0, 128256, 0.0), (1.0, 1, 0.0)])
@pytest.mark.parametrize("V", [128256, 259])
def test_sample_token_matches_upstream(temp, k, p, V):
    rng = np.random.default_rng(V + k)
    logits = Q.aligned_empty(V)
    if V < 1000:
        logits[:] = rng.standard_normal(V).astype(np.float32) * 3.0
    else:
        if k and 0.0 < p < 1.0:
            pytest.skip("upstream's top-p sort of the zeros top-k leaves degenerates on a large vocabulary")
        # every probability non-zero: logits within 1.8 temperatures of each other
        logits[:] = rng.uniform(-0.9, 0.9, V).astype(np.float32) * temp
    ours = in_fresh_thread(lambda: draws(Q.lib, logits, temp, k, p, 40))
    ref = in_fresh_thread(lambda: draws(O.ref, logits, temp, k, p, 40))
    assert ours == ref
    assert len(set(ours)) > 1 or k == 1  # it does draw, not always the argmax


@needs_ref
def test_sample_token_unaligned_logits_take_the_scalar_path():
    V = 1001
    rng = np.random.default_rng(7)
    raw = Q.aligned_empty(V + 1)
    raw[:] = rng.standard_normal(V + 1).astype(np.float32) * 2.0
    logits = raw[1:]  # 4 bytes past a 64-byte boundary
    assert logits.ctypes.data % 32 != 0
    ours = in_fresh_thread(lambda: draws(Q.lib, logits, 0.9, 50, 0.8, 30))
    ref = in_fresh_thread(lambda: draws(O.ref, logits, 0.9, 50, 0.8, 30))
    assert ours == ref


def test_sample_token_no_filter_is_valid():
    V = 5000
    logits = Q.aligned_empty(V)
    logits[:] = np.linspace(-3, 3, V, dtype=np.float32)
    toks = in_fresh_thread(lambda: draws(Q.lib, logits, 1.0, 0, 0.0, 200))
    assert all(0 <= t < V for t in toks)
    # the poly-exp softmax is zero more than ~2.5 below the max: only the top survives
    assert min(toks) > V - V // 10


@needs_ref
def test_q_generate_sampled_matches_upstream_loop(tiny_path, golden):
    """q_generate with temperature 0.9, top-k 20, top-p 0.9 on the device
    against upstream's loop (main.c:994-1131) run on the CPU: the upstream
    kernels' forward (oracle/_ref) and upstream q_sample_token."""
    prompt = np.ascontiguousarray(golden["tiny_prompt"], np.uint32)
    n = 24

    def ours():
        dev = Q.Model(tiny_path)
        tok = Q.q_tokenizer()
        tok.initialized = True
        tok.eos_token_id = 0xFFFFFFFF
        out = np.zeros(n, np.uint32)
        st = Q.q_generation_state()
        st.ctx = C.pointer(dev.ctx)
        st.model = C.pointer(dev.model)
        st.tokenizer = C.pointer(tok)
        st.prompt_tokens = prompt.ctypes.data_as(C.POINTER(C.c_uint32))
        st.num_prompt_tokens = len(prompt)
        st.generated_tokens = out.ctypes.data_as(C.POINTER(C.c_uint32))
        st.max_tokens = n
        st.temperature = 0.9
        st.top_k = 20
        st.top_p = 0.9
        Q.check(Q.lib.q_generate(C.byref(st)), "q_generate")
        assert st.num_generated_tokens == n
        # the thread's stream advanced once per token, as upstream's: the next
        # draw of this thread continues it
        lg = Q.aligned_empty(259)
        lg[:] = np.arange(259, dtype=np.float32) * 0.01
        nxt = draws(Q.lib, lg, 1.0, 0, 0.5, 1)
        dev.close()
        return list(out), nxt

    def upstream():
        m = O.RefModel(tiny_path)
        lg = Q.aligned_empty(259)
        lg[:] = m.forward(prompt, 0)
        toks = []
        pos = len(prompt)
        for _ in range(n):
            t = draws(O.ref, lg, 0.9, 20, 0.9, 1)[0]
            toks.append(t)
            lg[:] = m.forward(np.array([t], np.uint32), pos)
            pos += 1
        l2 = Q.aligned_empty(259)
        l2[:] = np.arange(259, dtype=np.float32) * 0.01
        nxt = draws(O.ref, l2, 1.0, 0, 0.5, 1)
        m.close()
        return toks, nxt

    a, an = in_fresh_thread(ours)
    b, bn = in_fresh_thread(upstream)
    assert a == b
    assert an == bn
