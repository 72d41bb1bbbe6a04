"""GPU: the checked build (libdsa_b200_checked.so, -DDSA_DEBUG_CHECKS).

Its guarded accesses test their index first and, on a failed test, set a bit
in a device flag word instead of accessing: no trap, no fault.  Each test runs
in a child process that loads the checked library (a process loads one
library), checks that a normal forward raises no flag and equals the normal
build's output bit for bit, and that a kept-index list holding entries past
the causal end is reported (bit 1) and those entries are left out.  The K/V
tensors are padded so that even an unchecked read of those entries would stay
inside their allocation."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CHECKED = os.path.join(REPO, "dsa-cpu-topk_b200", "libdsa_b200_checked.so")

CHILD = r"""
import json, math, os, sys, torch
sys.path[:0] = [os.path.join(REPO, "dsa-cpu-topk_b200"), os.path.join(REPO, "oracle")]
import _native, dsa_oracle as o
from dsa_attention import dsa_forward, sparse_attention_with_lists
out = {"enabled": int(_native.lib().dsa_debug_checks_enabled())}
dev = torch.device("cuda:0")
for dt in (torch.float32, torch.bfloat16):
    args = [x.to(dev) for x in o.make_inputs(2, 700, 8, 128, 4, 128, 128, dtype=dt)]
    O = dsa_forward(*args, 64)
    torch.save(O.cpu(), os.path.join(OUTDIR, "O_%s.pt" % str(dt).split(".")[-1]))
out["flags_forward"] = _native.debug_status()
# a kept-index list with entries past the causal end (and past T_k)
B, T, H, D = 1, 64, 2, 32
_, _, _, Q, K, V = o.make_inputs(B, T, 1, 8, H, D, D)
Kp = torch.zeros(B, T + 64, H, D); Kp[:, :T] = K
Vp = torch.zeros(B, T + 64, H, D); Vp[:, :T] = V
idx = torch.arange(8, dtype=torch.int32).repeat(T, 1)          # keys 0..7 for every row
cnt = torch.full((T,), 8, dtype=torch.int32)
idx[3, 5] = 40; idx[3, 6] = T + 10                             # row 3 (t=3): two keys past t
Qd, Kd, Vd = Q.to(dev), Kp.to(dev)[:, :T], Vp.to(dev)[:, :T]
sc = torch.zeros(B, T, T, device=dev); thr = torch.zeros(B * T, device=dev)   # unused: every cnt fits the list
res = sparse_attention_with_lists(idx.to(dev), cnt.to(dev), 8, sc, thr, Qd, Kd, Vd).cpu()
out["flags_list"] = _native.debug_status()
keep = [0, 1, 2, 3]                                             # row 3 keeps its causal keys 0..3 only
ref3 = o.attention_from_lists(keep, 4, Q, K, V, 0, 3)
out["row3_err"] = float((res[0, 3] - ref3).abs().max())
out["row10_err"] = float((res[0, 10] - o.attention_from_lists(list(range(8)), 8, Q, K, V, 0, 10)).abs().max())
print(json.dumps(out))
"""


def _run(variant, tmp_path):
    env = dict(os.environ, DSA_LIB_VARIANT=variant)
    code = "REPO = %r\nOUTDIR = %r\n" % (REPO, str(tmp_path / variant)) + CHILD
    os.makedirs(tmp_path / variant, exist_ok=True)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_checked_build_flags_bad_list_entries_and_matches_normal_build(cuda, tmp_path):
    import torch
    if not os.path.exists(CHECKED):
        pytest.fail("libdsa_b200_checked.so is not built (python dsa-cpu-topk_b200/build.py --checked)")
    chk = _run("checked", tmp_path)
    assert chk["enabled"] == 1
    assert chk["flags_forward"] == 0, chk
    assert chk["flags_list"] & 1, chk              # the out-of-range list entries were reported
    assert chk["row3_err"] < 1e-5 and chk["row10_err"] < 1e-5, chk
    for dt in ("float32", "bfloat16"):
        a = torch.load(tmp_path / "checked" / f"O_{dt}.pt")
        # the normal build on the same inputs, in this process
        import dsa_oracle as o
        from dsa_attention import dsa_forward
        tdt = getattr(torch, dt)
        args = [x.to(cuda) for x in o.make_inputs(2, 700, 8, 128, 4, 128, 128, dtype=tdt)]
        assert torch.equal(a, dsa_forward(*args, 64).cpu()), dt
