"""GPU: sf37_kvstore records written from device caches (sf37kv_kvstore_save)
against the record the reference's own store path writes for the same
session (sf37_kvstore_store_live_prefix_text on a CPU session, oracle/_ref),
and restored by sf37kv_kvstore_load with the reference's checks."""
import os
import tempfile

import numpy as np
import pytest
import torch

import oracle
from oracle import session as S
from tests import session_cases as C
from tests.test_oracle_session import _payload_src, _tie_only_diffs

pytestmark = pytest.mark.gpu
needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")
TEXT = "<|user|>What is the capital of France?<|assistant|>"


def _session(ctx, caps, kc, vc, toks, lg, hd):
    from sf37_b200.session import Session
    s = Session(ctx, [(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()) for k, v in zip(kc, vc)])
    s.set_tokens(toks)
    s.logits[:] = lg
    s.hidden[:] = hd
    return s


@needs_ref
@pytest.mark.parametrize("ctx,n", [(48, 40), (600, 530)])
def test_record_matches_reference_store(ctx, n):
    caps = [ctx] * C.LAYERS
    toks, lg, hd, kc, vc = C.state(11, ctx, n, caps)
    rows = S.layer_rows(n, ctx, caps)
    krows = [C.live_rows_in_order(kc[il], n, rows[il], caps[il]) for il in range(C.LAYERS)]
    vrows = [C.live_rows_in_order(vc[il], n, rows[il], caps[il]) for il in range(C.LAYERS)]
    with tempfile.TemporaryDirectory() as d:
        ref = S.ref_kvstore_store(d, ctx, toks, lg, hd, krows, vrows, TEXT)
    created = int.from_bytes(ref[24:32], "little")
    s = _session(ctx, caps, kc, vc, toks, lg, hd)
    with tempfile.TemporaryFile() as f:
        nb = s.kvstore_save(f, TEXT, reason=1, now=created)
        f.seek(0)
        mine = f.read()
    assert nb == len(mine) == len(ref)
    # header and text exactly; the payload up to the reference encoder's
    # CPU-specific .5 ties (see _tie_only_diffs)
    head = 52 + len(TEXT)
    assert mine[:head] == ref[:head]
    # payload header word 10 is the backend kind (sf37.c:6942): 1 for a
    # session on CUDA caches, 0 for the reference's CPU session
    w10 = head + 40
    assert mine[w10:w10 + 4] == (1).to_bytes(4, "little") and ref[w10:w10 + 4] == bytes(4)
    mine = mine[:w10] + bytes(4) + mine[w10 + 4:]
    _tie_only_diffs(mine[head:], ref[head:], (15 + C.LAYERS + n + C.VOCAB + C.EMBD) * 4,
                    _payload_src(kc, vc, n, ctx, caps))


def test_record_roundtrip_and_checks():
    from sf37_b200.session import SessionError
    ctx, n = 600, 530
    caps = [ctx if il % 4 == 0 else 520 for il in range(C.LAYERS)]
    toks, lg, hd, kc, vc = C.state(12, ctx, n, caps, f16=True)
    from sf37_b200.session import Session
    k = [torch.from_numpy(a.view(np.float16)).cuda() for a in kc]
    v = [torch.from_numpy(a.view(np.float16)).cuda() for a in vc]
    s = Session(ctx, list(zip(k, v)))
    s.set_tokens(toks)
    s.logits[:] = lg
    s.hidden[:] = hd
    import hashlib
    sha = hashlib.sha1(TEXT.encode()).hexdigest()
    with tempfile.TemporaryFile() as f:
        f.write(b"xyz")  # records start at the descriptor's offset
        s.kvstore_save(f, TEXT, now=5)
        blank = [(torch.zeros_like(a), torch.zeros_like(b)) for a, b in zip(k, v)]
        r = Session(ctx, blank)
        f.seek(3)
        assert r.kvstore_load(f, TEXT + " Paris?", sha) == n
        # the payload rows are int8-grouped (lossy): the restored slots equal
        # the oracle's decode of the same payload bytes
        f.seek(3 + 52 + len(TEXT))
        ok_k = [np.zeros_like(a) for a in kc]
        ok_v = [np.zeros_like(a) for a in vc]
        S.load(1, f.read(), ctx, caps, ok_k, ok_v)
        for il in range(C.LAYERS):
            rows = min(n, caps[il])
            slots = [(n - rows + i) % caps[il] for i in range(rows)]
            gk = blank[il][0].cpu().numpy().view(np.uint16)
            gv = blank[il][1].cpu().numpy().view(np.uint16)
            assert np.array_equal(gk[slots], ok_k[il][slots])
            assert np.array_equal(gv[slots], ok_v[il][slots])
        assert np.array_equal(r.tokens[:n], toks)
        for prompt, key, msg in (("What", sha, "cached text is longer than prompt"),
                                 ("<|user|>What is the capital of Sweden?<|assistant|>", sha,
                                  "cached text prefix mismatch"),
                                 (TEXT, "0" * 40, "cached text hash mismatch")):
            f.seek(3)
            with pytest.raises(SessionError, match=msg):
                r.kvstore_load(f, prompt, key)
        f.seek(0)
        with pytest.raises(SessionError, match="invalid header"):
            r.kvstore_load(f, TEXT, sha)
