"""Generates the golden fixtures in this folder from the REFERENCE's own PyTorch code.

Run once, in a container where the reference repository is importable:

    python tests/golden/make_golden.py /path/to/Tilelang-FA-V100

It imports ``pytorch_gqa_ref`` and ``make_paged_gqa`` from the reference's
tests/test_gqa_paged.py (the module is importable on CPU; its ``main`` is not run)
and evaluates them on CPU.  Cases are the reference's own parity cases
(test_gqa_paged.py:229-246, 260-268: GQA prefill, chunked prefill) plus dense MHA
cases in the shape family of tests/test_compare_ref.py:43-52, a non-square causal
case, scattered pages and a decode case (q_len = 1).  Inputs follow the reference
convention (torch.manual_seed(42), torch.randn fp16).  Stored per case: inputs,
the reference's fp16 output, the LSE of the same scores (torch.logsumexp; the
reference oracle itself returns no LSE) and, for dense cases, the gradients from
torch autograd through ``pytorch_gqa_ref`` for an N(0,1) dO.

Nothing at test time reads the reference; the tests only load the .npz files.
"""
import importlib.util
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(root):
    path = os.path.join(root, "tests", "test_gqa_paged.py")
    spec = importlib.util.spec_from_file_location("ref_test_gqa_paged", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def lse_of(q, k, causal):
    b, hq, m, d = q.shape
    hkv, n = k.shape[1], k.shape[2]
    ke = k.float().repeat_interleave(hq // hkv, dim=1)
    s = torch.einsum("bhqd,bhkd->bhqk", q.float(), ke) / math.sqrt(d)
    if causal:
        mask = torch.tril(torch.ones(m, n), diagonal=n - m)
        s = s.masked_fill(mask == 0, float("-inf"))
    return torch.logsumexp(s, dim=-1)


def dense_case(ref, name, b, hq, hkv, m, n, d, causal, with_grad=True):
    torch.manual_seed(42)
    q = torch.randn(b, hq, m, d, dtype=torch.float16)
    k = torch.randn(b, hkv, n, d, dtype=torch.float16)
    v = torch.randn(b, hkv, n, d, dtype=torch.float16)
    out = ref.pytorch_gqa_ref(q, k, v, causal)
    rec = dict(q=q.numpy(), k=k.numpy(), v=v.numpy(), out=out.numpy(),
               lse=lse_of(q, k, causal).numpy().astype(np.float32),
               causal=np.array(causal))
    if with_grad:
        do = torch.randn(b, hq, m, d, dtype=torch.float32)
        qf = q.float().requires_grad_(True)
        kf = k.float().requires_grad_(True)
        vf = v.float().requires_grad_(True)
        o = ref.pytorch_gqa_ref(qf, kf, vf, causal).float()
        o.backward(do)
        rec.update(do=do.numpy(), dq=qf.grad.numpy(), dk=kf.grad.numpy(), dv=vf.grad.numpy())
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)
    print("wrote", name)


def paged_case(ref, name, b, hq, hkv, m, n, d, causal, shuffle_seed=None):
    """Prefill (m == n) or chunked prefill (m < n, prefix = n - m) through make_paged_gqa."""
    torch.manual_seed(42)
    if m == n:
        q = torch.randn(b, hq, m, d, dtype=torch.float16)
        k = torch.randn(b, hkv, n, d, dtype=torch.float16)
        v = torch.randn(b, hkv, n, d, dtype=torch.float16)
    else:  # order of draws as in test_gqa_chunked_prefill (test_gqa_paged.py:161-165)
        k = torch.randn(b, hkv, n, d, dtype=torch.float16)
        v = torch.randn(b, hkv, n, d, dtype=torch.float16)
        q = torch.randn(b, hq, m, d, dtype=torch.float16)
    out = ref.pytorch_gqa_ref(q, k, v, causal)
    pd = ref.make_paged_gqa(q, k, v, page_block_size=16)
    kc, vc, bt = pd["K_cache"], pd["V_cache"], pd["block_table"]
    if m != n:
        # make_paged_gqa pages the first m tokens only; chunked prefill pages all n
        # exactly as test_gqa_chunked_prefill does (test_gqa_paged.py:176-199).
        pps = math.ceil(n / 16)
        kc = torch.zeros(b * pps, 16, hkv, d, dtype=torch.float16)
        vc = torch.zeros(b * pps, 16, hkv, d, dtype=torch.float16)
        for bb in range(b):
            for t in range(n):
                kc[bb * pps + t // 16, t % 16] = k[bb, :, t]
                vc[bb * pps + t // 16, t % 16] = v[bb, :, t]
        bt = torch.arange(b * pps, dtype=torch.int32).reshape(b, pps)
    if shuffle_seed is not None:
        g = torch.Generator().manual_seed(shuffle_seed)
        perm = torch.randperm(kc.shape[0], generator=g)
        kc2 = torch.zeros_like(kc)
        vc2 = torch.zeros_like(vc)
        kc2[perm] = kc
        vc2[perm] = vc
        kc, vc, bt = kc2, vc2, perm[bt.long()].to(torch.int32)
    qsl = torch.arange(0, (b + 1) * m, m, dtype=torch.int32)
    rec = dict(q_flat=q.permute(0, 2, 1, 3).reshape(b * m, hq, d).numpy(), k_cache=kc.numpy(),
               v_cache=vc.numpy(), block_table=bt.numpy(),
               seq_lens=np.full((b,), n, np.int32), query_start_loc=qsl.numpy(),
               prefix_kv_lens=np.full((b,), n - m, np.int32),
               out=out.permute(0, 2, 1, 3).reshape(b * m, hq, d).numpy(),
               lse=lse_of(q, k, causal).permute(1, 0, 2).reshape(hq, b * m).numpy(),
               causal=np.array(causal))
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)
    print("wrote", name)


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REFERENCE_ROOT", "")
    ref = load_reference(root)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    # dense MHA (shape family of test_compare_ref.py:43-52) and a non-square causal case
    dense_case(ref, "dense_mha_d64_noncausal", 1, 2, 2, 96, 96, 64, False)
    dense_case(ref, "dense_mha_d64_causal", 1, 2, 2, 96, 96, 64, True)
    dense_case(ref, "dense_mha_d128_causal", 1, 2, 2, 80, 80, 128, True)
    dense_case(ref, "dense_nonsquare_causal", 1, 2, 2, 40, 104, 128, True)
    dense_case(ref, "dense_gqa_d128", 1, 4, 2, 48, 48, 128, True)
    # paged GQA prefill (test_gqa_paged.py:235-242) and chunked prefill (:264-267)
    paged_case(ref, "paged_gqa_16_2_d128", 1, 16, 2, 64, 64, 128, True)
    paged_case(ref, "paged_gqa_24_4_d128", 1, 24, 4, 64, 64, 128, True)
    paged_case(ref, "paged_gqa_4_1_d128", 1, 4, 1, 64, 64, 128, True)
    paged_case(ref, "paged_gqa_8_1_d256", 1, 8, 1, 64, 64, 256, True)
    paged_case(ref, "paged_gqa_noncausal_d256", 1, 8, 1, 64, 64, 256, False)
    paged_case(ref, "paged_chunked_16_2_d128", 1, 16, 2, 32, 128, 128, True)
    paged_case(ref, "paged_chunked_8_1_d256", 1, 8, 1, 16, 64, 256, True)
    paged_case(ref, "paged_multibatch_shuffled", 2, 16, 2, 48, 48, 128, True, shuffle_seed=7)
    # decode: one query token per sequence attends to every key
    paged_case(ref, "decode_gqa_16_4_d128", 3, 16, 4, 1, 100, 128, True, shuffle_seed=3)
    # decode at the reference's synthetic 8/1 D=256 configuration (test_gqa_paged.py:239-240)
    paged_case(ref, "decode_gqa_8_1_d256", 2, 8, 1, 1, 200, 256, True, shuffle_seed=5)


if __name__ == "__main__":
    main()
