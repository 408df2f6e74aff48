"""Test harness: the same pool built on the GPU (through the C-ABI) and in
the CPU oracle, driven with identical synthetic inputs."""
from __future__ import annotations

import numpy as np

TOL_ABS, TOL_REL = 1e-4, 1e-3  # north_star tolerance for fp32 attention outputs


def assert_close(gpu, ref, what=""):
    gpu = np.asarray(gpu, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(gpu - ref)
    bound = TOL_ABS + TOL_REL * np.abs(ref)
    bad = err > bound
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} outside |d| <= 1e-4 + 1e-3|ref|; "
                           f"max err {err.max():.3e}")


class Twin:
    """A GPU KvPool and an oracle Pool with the same geometry and history."""

    def __init__(self, torch, codec, layers, kv_heads, page_tokens, total_pages, max_seqs, max_pages,
                 query_heads, perm_seed=0, seed=1):
        import qwanto_b200 as qb
        from oracle import oracle as O
        self.torch, self.qb, self.O = torch, qb, O
        self.codec, self.layers, self.HK, self.P = codec, layers, kv_heads, page_tokens
        self.H, self.seed = query_heads, seed
        self.gpu = qb.KvPool(codec, layers, kv_heads, page_tokens, total_pages, max_seqs, max_pages,
                             max_query_heads=query_heads, permutation_seed=perm_seed)
        self.ora = O.Pool(codec, layers, kv_heads, page_tokens, total_pages, max_seqs, max_pages,
                          perm_seed=perm_seed)
        self.mask = None  # optional [layers][HK*128] outlier mask

    def close(self):
        self.gpu.close()

    def row(self, kind, seq, layer, pos, width):
        r = self.O.gen_row(self.seed, kind, seq, layer, pos, width)
        if kind == 2 and self.mask is not None:
            r = np.where(self.mask[layer] != 0, r * np.float32(8), r).astype(np.float32)
        return r

    def prefill(self, seq_ids, lens):
        self.gpu.prefill_synthetic(seq_ids, lens, self.seed, self.mask)
        assert self.ora.append(seq_ids, lens) == 0
        W = self.HK * 128
        for s, n in zip(seq_ids, lens):
            for layer in range(self.layers):
                for t in range(n):
                    assert self.ora.write(s, layer, t, self.row(2, s, layer, t, W), self.row(3, s, layer, t, W)) == 0

    def step(self, seq_ids, page_mass=False, identity=False):
        """One decode step on both sides: grow each listed sequence by one
        token, then per layer append + attend.  Returns (gpu, oracle) outputs
        [layers][n][H][128] and, with page_mass, the per-page mass arrays.
        identity: seq_ids is 0..n-1 and the GPU calls pass no id array (the
        form whose launch setup is cached across the layers of a step)."""
        torch, qb = self.torch, self.qb
        n = len(seq_ids)
        if identity:
            assert list(seq_ids) == list(range(n))
        ids = torch.tensor(seq_ids, dtype=torch.int32, device="cuda")
        self.gpu.seq_append(n, None if identity else ids)
        assert self.ora.append(seq_ids, [1] * n) == 0
        pos_host = np.array([int(self.ora.lens()[s]) - 1 for s in seq_ids], np.int32)
        pos = torch.tensor(pos_host, device="cuda")
        W, Wq = self.HK * 128, self.H * 128
        outs_g, outs_o, masses = [], [], []
        mask_dev = None
        for layer in range(self.layers):
            q = torch.empty((n, Wq), dtype=torch.float32, device="cuda")
            k = torch.empty((n, W), dtype=torch.float32, device="cuda")
            v = torch.empty((n, W), dtype=torch.float32, device="cuda")
            if self.mask is not None:
                mask_dev = torch.tensor(self.mask[layer], device="cuda")
            qb.generate_rows(q, n, Wq, 1, self.seed, layer, ids, pos)
            qb.generate_rows(k, n, W, 2, self.seed, layer, ids, pos, mask_dev)
            qb.generate_rows(v, n, W, 3, self.seed, layer, ids, pos)
            out = torch.zeros((n, Wq), dtype=torch.float32, device="cuda")
            pm = None
            if page_mass:
                pm = torch.zeros((self.gpu.max_seqs, self.gpu.max_pages_per_seq), dtype=torch.float32,
                                 device="cuda")
            self.gpu.decode(layer, n, self.H, q, out, key=k, value=v, seq_ids=None if identity else ids,
                            page_mass=pm)
            torch.cuda.synchronize()
            res_o = np.zeros((n, self.H, 128), np.float32)
            for i, s in enumerate(seq_ids):
                p = int(pos_host[i])
                assert self.ora.write(s, layer, p, self.row(2, s, layer, p, W), self.row(3, s, layer, p, W)) == 0
                res_o[i] = self.ora.attention(s, layer, p + 1, self.row(1, s, layer, p, Wq), self.H,
                                              1.0 / np.sqrt(128.0))
            outs_g.append(out.cpu().numpy().reshape(n, self.H, 128))
            outs_o.append(res_o)
            if page_mass:
                masses.append(pm.cpu().numpy())
        return np.stack(outs_g), np.stack(outs_o), masses

    def assert_state_equal(self):
        g, o = self.gpu, self.ora
        assert np.array_equal(g.lens(), o.lens())
        assert np.array_equal(g.npages(), o.npages())
        assert np.array_equal(g.page_table(), o.page_table())
        assert np.array_equal(g.free_stack(), o.free_stack())

    def assert_pages_equal(self):
        used = sorted({int(x) for x in self.ora.page_table().ravel() if x >= 0})
        pages_o = self.ora.pages()
        for pg in used:
            a, b = self.gpu.page(pg), pages_o[pg]
            if not np.array_equal(a, b):
                diff = np.nonzero(a != b)[0]
                raise AssertionError(f"page {pg}: {diff.size} bytes differ, first at {diff[:8]}")
