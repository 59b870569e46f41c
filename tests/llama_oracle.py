"""CPU model of the Llama-shaped family built on the oracle (test infrastructure).

Weights come from the same counter-based generator as clm_b200_engine_generate_weights (tensor id
16*layer + {q,k,v,o,gate,up,down}; 1000 embedding; 1001 head; 1002..1004 MTP gate/up/down), encoded by the
oracle's encoders, so the device engine and this model hold identical bytes.
"""
from __future__ import annotations

import numpy as np

from oracle.oracle_py import LlamaDims, Oracle


class LlamaOracle:
    def __init__(self, orc: Oracle, geo, seed: int = 0, stddev: float = 0.02, layers=None, max_ctx: int = 256,
                 threads: int = 8):
        self.o, self.g, self.seed, self.std, self.threads = orc, geo, seed, stddev, threads
        H, nh, nkv, hd, F, V = geo.hidden, geo.n_heads, geo.n_kv_heads, geo.head_dim, geo.ffn, geo.vocab
        self.dims = LlamaDims(H, nh, nkv, hd, F, geo.rope_theta, geo.rms_eps)
        self.q = geo.quant
        self.layers = list(range(geo.n_layers)) if layers is None else list(layers)
        qd, kvd = nh * hd, nkv * hd
        self.w = {}
        for L in self.layers:
            i = 16 * L
            self.w[L] = (
                np.concatenate([self.enc(i + 0, qd * H), self.enc(i + 1, kvd * H), self.enc(i + 2, kvd * H)]),
                self.enc(i + 3, H * qd),
                np.concatenate([self.enc(i + 4, F * H), self.enc(i + 5, F * H)]),
                self.enc(i + 6, H * F),
            )
        self.ones = np.ones(H, np.float32)
        self.kc = {L: np.zeros((max_ctx, kvd), np.float32) for L in self.layers}
        self.vc = {L: np.zeros((max_ctx, kvd), np.float32) for L in self.layers}
        self._head = None

    def enc(self, tensor_id: int, n: int) -> np.ndarray:
        chunk = 1 << 22  # whole Q4_K superblocks / Q8_0 blocks; chunks are generated and encoded on all threads
        if n <= chunk:
            return self.o.encode(self.q, self.o.gen_weights(self.seed, tensor_id, 0, n, self.std))
        import concurrent.futures as cf

        with cf.ThreadPoolExecutor(max_workers=self.threads) as pool:
            parts = list(pool.map(
                lambda f: self.o.encode(self.q, self.o.gen_weights(self.seed, tensor_id, f, min(chunk, n - f),
                                                                   self.std)), range(0, n, chunk)))
        return np.concatenate(parts)

    @property
    def head(self):
        if self._head is None:
            self._head = self.enc(1001, self.g.vocab * self.g.hidden)
        return self._head

    def embed(self, tokens) -> np.ndarray:
        """Embedding rows, generated and encoded row by row (a row is whole blocks, so its bytes are the full
        table's bytes of that row)."""
        H = self.g.hidden
        return np.stack([self.o.decode(self.q, self.o.encode(self.q, self.o.gen_weights(
            self.seed, 1000, int(t) * H, H, self.std)), H) for t in tokens])

    def fill_context(self, tokens) -> None:
        """K / V rows of positions 0..len(tokens)-1 in every layer, as a prefill of `tokens` writes them; only the
        first layer's rows are exact without running the layers, so this is for single-layer models."""
        assert len(self.layers) == 1, "fill_context computes the first layer's caches only"
        L = self.layers[0]
        h = self.embed(tokens)
        self.o.llama_kv_rows(self.dims, self.q, self.w[L][0], self.ones, self.kc[L], self.vc[L], 0, h, self.threads)

    def run_layers(self, h: np.ndarray, base: int, parent=None) -> np.ndarray:
        h = np.ascontiguousarray(h, np.float32).copy()
        for L in self.layers:
            wqkv, wo, wgu, wd = self.w[L]
            self.o.llama_layer(self.dims, self.q, wqkv, wo, wgu, wd, self.ones, self.ones, self.kc[L], self.vc[L],
                               base, h, parent, self.threads)
        return h

    def logits(self, h: np.ndarray) -> np.ndarray:
        x = np.stack([self.o.rmsnorm(r, self.ones, self.g.rms_eps) for r in h])
        return self.o.matmul_rows_quant(self.q, self.head, self.g.vocab, self.g.hidden, x, self.threads)

    def window(self, tokens, base: int) -> np.ndarray:
        return self.logits(self.run_layers(self.embed(tokens), base))

    def mtp_logits(self, prev: int) -> np.ndarray:
        g = self.g
        if not hasattr(self, "_mtp"):
            self._mtp = (np.concatenate([self.enc(1002, g.ffn * g.hidden), self.enc(1003, g.ffn * g.hidden)]),
                         self.enc(1004, g.hidden * g.ffn))
        gu, down = self._mtp
        x = self.embed([prev])
        xn = self.o.rmsnorm(x[0], self.ones, g.rms_eps)[None]
        y = self.o.matmul_rows_quant(self.q, gu, 2 * g.ffn, g.hidden, xn, self.threads)[0]
        a = np.array([self.o.L.orc_silu(float(v)) for v in y[:g.ffn]], np.float32) * y[g.ffn:]
        d = self.o.matmul_rows_quant(self.q, down, g.hidden, g.ffn, a[None], self.threads)[0]
        return self.logits((x[0] + d)[None])[0]
