"""C1 end to end with the KV cache on the GPU.

The forward pass is the oracle's CPU restatement of model.rs:366-518 (Q8_0
Llama, 22 layers, hidden 2048, 32/4 heads, head_dim 64, FFN 5632, vocab
32000, seed 0).  Its KV cache is the GPU cache, driven through the C ABI
with every call mirrored on an oracle KvCache:
- every append returns the oracle's (block, slot), bit-exact;
- every attention output is within max-abs 2e-3 / rel 1e-3 of the oracle's
  attention on the same q (per layer, per call);
- after the run the GPU pool, tables, refcounts and free list equal the
  oracle's, bit-exact;
- the 4 x 64 greedy tokens equal those of the all-oracle run.
"""
import numpy as np
import pytest
import torch

from oracle import model as M

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-3


class _GpuTwinKv:
    def __init__(self, oracle_mod, m, n_tokens, max_seqs):
        from langtrain_studio_b200.kv import KvCache

        self.m = m
        self.kv = KvCache(m.n_layers, m.n_kv_heads, m.head_dim, n_tokens, n_heads=m.n_heads, max_seqs=max_seqs,
                          max_batch=512, device=0)
        self.ok = oracle_mod.OracleKv(m.n_layers, m.kv_dim, n_tokens, max_seqs=max_seqs)
        self.max_seqs = max_seqs
        self.worst = 0.0  # max |gpu - ref| / (ATOL + RTOL |ref|) over all calls
        self.calls = 0

    def append(self, seqs, pos):
        b, s = self.kv.append_batch(seqs, pos)
        rc, done, bo, so = self.ok.append_batch(seqs, pos)
        assert rc == 0 and np.array_equal(b, bo) and np.array_equal(s, so)
        return b, s

    def write(self, layer, b, s, k, v):
        self.kv.write(layer, b, s, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
        self.ok.write_batch(layer, b, s, k, v)

    def attend(self, layer, q, seqs, pos):
        out = self.kv.attend(layer, torch.from_numpy(q).cuda(), seqs, pos).cpu().numpy()
        ref = self.ok.attend(layer, q, seqs, pos, self.m.n_heads, self.m.n_kv_heads, self.m.head_dim)
        r = float((np.abs(out - ref) / (ATOL + RTOL * np.abs(ref))).max())
        self.worst = max(self.worst, r)
        self.calls += 1
        assert r <= 1.0, f"layer {layer}: attention outside tolerance (ratio {r:.3f})"
        return out

    def share(self, src, dst, n):
        self.kv.share(src, dst, n)
        self.ok.share(src, dst, n)

    def check_state(self):
        torch.cuda.synchronize()
        ko, vo = self.ok.pool()
        for layer in range(self.m.n_layers):
            k, v = self.kv.pool_reference_layout(layer)
            assert np.array_equal(k, ko[layer]) and np.array_equal(v, vo[layer]), f"pool differs in layer {layer}"
        assert np.array_equal(self.kv.free_list(), self.ok.free_list())
        assert np.array_equal(self.kv.refs(), self.ok.refs())
        for s in range(self.max_seqs):
            assert np.array_equal(self.kv.seq_blocks(s), self.ok.seq_blocks(s))


def test_c1_end_to_end_greedy_tokens(oracle_mod):
    assert torch.cuda.is_available(), "CUDA device required"
    m = M.OracleModel(**M.C1_SHAPE, seed=0)
    prompts = M.c1_prompts(m.vocab)
    ref_kv = m.oracle_kv(1024, 4)
    ref = M.run_c1(m, ref_kv, ref_kv.share, prompts, 64, 64)
    twin = _GpuTwinKv(oracle_mod, m, 1024, 4)
    got = M.run_c1(m, M.PyKv(twin, m.kv_dim, m.q_dim), twin.share, prompts, 64, 64)
    twin.check_state()
    assert twin.calls == m.n_layers * 65
    assert np.array_equal(got, ref), f"greedy tokens differ at {np.argwhere(got != ref)[:8].tolist()}"
    print(f"C1: {got.size} tokens identical; worst attention error {twin.worst:.3f} of tolerance")
