"""Generates the golden fixtures in this directory from the REFERENCE's own
CPU code (oracle/_ref/libsf37ref.so, compiled from the reference sources with
its Makefile flags by `make -C oracle ref`).  Run in the development
container where the reference tree exists:

    python tests/golden/make_golden.py

Fixtures (all inputs are regenerable from the seeds in sf37_b200.synth):
  payload_rows.npz  16 N(0,1)*3 rows + the reference self-test pattern row +
                    a zero row, and their int8-grouped encodings (group 64)
  cfg1_decode.npz   BASELINE config 1 (2048 f16-valued rows + 1 appended
                    fp32 row, 64 Q / 8 KV heads, d 128): attention_decode
                    output without and with the sigmoid gate
  sliding_decode.npz 96 Q heads (group 12), 600 rows, sliding window 512
  kv_push.npz       kv_cache_push of 6 rows into a capacity-4 linear cache
  sessions.npz      session snapshot / payload bytes and loader messages
                    (see sessions() below)
  q8_0.npz          sf37_q8_0_quantize_activation of an 8192-element x (with
                    a zero block) and sf37_q8_0_matvec of 16 rows of Q8_0
                    weights (sf37_b200.synth.q8_0_weights(31, 16, 8192))
  qk_prep.npz       head_rms_norm_weight1 + apply_rope_one on 9 heads at 6
                    positions, full-layer (64, 5e6, llama3) and sliding-layer
                    (128, 1e4) parameters
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
import oracle  # noqa: E402
from sf37_b200 import synth  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def main():
    assert oracle.ref_available(), "build oracle/_ref first: make -C oracle ref"
    # payload rows
    rows = synth.normal(101, (16, 1024)) * np.float32(3.0)
    pat = ((np.arange(1024) % 97).astype(np.int32) - 48).astype(np.float32) / np.float32(13.0)
    rows = np.vstack([rows, pat[None], np.zeros((1, 1024), np.float32)]).astype(np.float32)
    enc = oracle.ref_payload_encode_rows(rows)
    dec = oracle.ref_payload_decode_rows(enc, 1024)
    np.savez_compressed(os.path.join(OUT, "payload_rows.npz"), rows=rows, enc=enc, dec=dec)

    # config 1
    k, v, k_new, v_new, q, gate = synth.cfg1_inputs(0)
    cap = 2049
    kc = np.zeros((cap, 1024), np.float32)
    vc = np.zeros((cap, 1024), np.float32)
    n = oracle.ref_kv_cache_push(kc, vc, cap, 0, k.astype(np.float32), v.astype(np.float32))
    n = oracle.ref_kv_cache_push(kc, vc, cap, n, k_new[None], v_new[None])
    out_nogate = oracle.ref_attention_decode(q, kc, vc, n, cap, 64, 0, None)
    out_gate = oracle.ref_attention_decode(q, kc, vc, n, cap, 64, 0, gate)
    np.savez_compressed(os.path.join(OUT, "cfg1_decode.npz"), out_nogate=out_nogate,
                        out_gate=out_gate, n_live=n)

    # sliding layer of the real model: 96 query heads, window 512
    ks = synth.normal(201, (600, 1024))
    vs = synth.normal(202, (600, 1024))
    qs = synth.normal(203, (96, 128))
    gs = synth.normal(204, (96,))
    out_s = oracle.ref_attention_decode(qs, ks, vs, 600, 600, 96, 1, gs)
    np.savez_compressed(os.path.join(OUT, "sliding_decode.npz"), out=out_s)

    # kv_cache_push wrap behaviour (memmove when full)
    kp = synth.normal(301, (6, 1024))
    vp = synth.normal(302, (6, 1024))
    kc4 = np.zeros((4, 1024), np.float32)
    vc4 = np.zeros((4, 1024), np.float32)
    n4 = oracle.ref_kv_cache_push(kc4, vc4, 4, 0, kp, vp)
    np.savez_compressed(os.path.join(OUT, "kv_push.npz"), k=kc4, v=vc4, n=n4)
    print("golden fixtures written to", OUT)



def sessions():
    """sessions.npz: the reference's own sf37_session_save_snapshot and
    sf37_session_save_payload on a CPU session (ctx 3, 2 tokens, values on a
    1/2 grid), and the message its loaders give for each corruption in
    tests/session_cases.py (both loaders, on the reference's own bytes)."""
    from oracle import session as S
    from tests import session_cases as C
    ctx, n = 3, 2
    toks, lg, hd, kc, vc = C.state(7, ctx, n, [ctx] * C.LAYERS, coarse=True)
    rows = S.layer_rows(n, ctx, [ctx] * C.LAYERS)
    kr = [C.live_rows_in_order(kc[i], n, rows[i], ctx) for i in range(C.LAYERS)]
    vr = [C.live_rows_in_order(vc[i], n, rows[i], ctx) for i in range(C.LAYERS)]
    snap = S.ref_session_save(0, ctx, toks, lg, hd, kr, vr)
    pay = S.ref_session_save(1, ctx, toks, lg, hd, kr, vr)
    names, msgs = [], []
    for kind, buf in ((0, snap), (1, pay)):
        for name, bad, lctx in C.corruptions(kind, buf, ctx):
            try:
                S.ref_session_load(kind, bad, lctx)
                msg = ""
            except S.LoadError as e:
                msg = str(e)
            names.append(f"{kind}:{name}")
            msgs.append(msg)
    np.savez_compressed(os.path.join(OUT, "sessions.npz"), snapshot=np.frombuffer(snap, np.uint8),
                        payload=np.frombuffer(pay, np.uint8), names=np.array(names), msgs=np.array(msgs))


def q8_0():
    x = synth.normal(30, (8192,)) * 2
    x[64:96] = 0
    w = synth.q8_0_weights(31, 16, 8192)
    xq, xs = oracle.ref_q8_0_quantize(x)
    out = oracle.ref_q8_0_matvec(w, x, 16)
    np.savez_compressed(os.path.join(OUT, "q8_0.npz"), xq=xq, xs=xs, out=out)


QK_POS = (0, 1, 511, 4097, 32768, 131071)


def qk_prep():
    rng = np.random.default_rng(21)
    x = (rng.standard_normal((len(QK_POS), 9, 128)) * 3).astype(np.float32)
    w = ((rng.standard_normal(128) * 0.3).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    full = np.stack([oracle.ref_qk_prep(x[i], w, 64, 5e6, 1, p) for i, p in enumerate(QK_POS)])
    sliding = np.stack([oracle.ref_qk_prep(x[i], w, 128, 1e4, 0, p) for i, p in enumerate(QK_POS)])
    np.savez_compressed(os.path.join(OUT, "qk_prep.npz"), x=x, w=w, pos=np.array(QK_POS), full=full,
                        sliding=sliding)


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "sessions":
        sessions()
    elif len(sys.argv) > 1 and sys.argv[1] == "qk_prep":
        qk_prep()
    elif len(sys.argv) > 1 and sys.argv[1] == "q8_0":
        q8_0()
    else:
        main()
        sessions()
        qk_prep()
        q8_0()
