"""Generates the golden vectors under tests/golden/ by running the REFERENCE's own code.

Run in a container that has the reference sources (oracle/_ref/libclm_ref.so is compiled from them by
oracle/Makefile) and gguf-py 0.19.0:

    python tests/golden/make_golden.py

Outputs (numpy .npz, committed):
  codec.npz     binary16 conversions, q8_0 / q8_0-fixture encode+decode (reference tensor_codec.cpp),
                Q4_K blocks from the oracle encoder decoded by gguf-py (the Q4_K pin)
  sampling.npz  distribution / sample_from / verify_speculative outcomes (reference sampling.cpp)
  philox.npz    Philox4x32-10 known-answer vectors (Random123 kat_vectors) and derived uniforms
  fixture.npz   reference fixture model (default spec), plan 0-4/4-10/10-13/13-16, greedy and q=4
                scripted:0.3 speculative generation: per-window tokens, accepted counts and logits
"""
from __future__ import annotations

import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle_py import Oracle, Reference, RefPipeline  # noqa: E402

FIXTURE_SEED = 0x434C4D31
PLAN_BOUNDS = [0, 4, 10, 13, 16]


def make_codec(ref: Reference, orc: Oracle) -> dict:
    rng = np.random.default_rng(1234)
    out = {}
    hs = np.arange(0, 0x10000, 7, dtype=np.uint32)
    out["h2f_in"] = hs.astype(np.uint16)
    out["h2f_out"] = np.array([ref.L.ref_half_to_float(int(h)) for h in hs], np.float32)
    fs = np.concatenate([
        rng.standard_normal(2000).astype(np.float32) * 100,
        (rng.standard_normal(1000) * 1e-5).astype(np.float32),
        np.array([0.0, -0.0, 1.0, -2.0, 65504.0, 65520.0, 1e10, -1e10, 6.103515625e-05, 5.960464477539063e-08,
                  1.0 + 1.0 / 2048.0, 1.0 + 3.0 / 2048.0, np.inf, -np.inf], np.float32),
    ])
    out["f2h_in"] = fs
    out["f2h_out"] = np.array([ref.L.ref_float_to_half(float(f)) for f in fs], np.uint16)
    v = (rng.standard_normal(64 * 32) * np.repeat(np.arange(1, 65), 32) * 0.01).astype(np.float32)
    v[32:64] = 0.0  # an all-zero block
    out["q8_in"] = v
    for name, key in (("q8_0", "q8_0"), ("q8_0-fixture", "q8f")):
        enc = ref.encode(name, v)
        out[f"{key}_bytes"] = enc
        out[f"{key}_decoded"] = ref.decode(name, enc, v.size)
    import gguf
    from gguf import quants

    w = (rng.standard_normal(256 * 48) * 0.02).astype(np.float32)
    w[256:512] = np.abs(w[256:512])  # a superblock with no negative values (min clamps to 0)
    w[512:768] = 0.0                 # an all-zero superblock
    enc = orc.encode("q4_k", w)
    out["q4k_in"] = w
    out["q4k_bytes"] = enc
    out["q4k_decoded_gguf"] = quants.dequantize(enc.reshape(-1, 144), gguf.GGMLQuantizationType.Q4_K).reshape(-1)
    return out


def make_sampling(ref: Reference) -> dict:
    rng = np.random.default_rng(99)
    V = 1000
    out = {"V": np.int32(V)}
    logits = (rng.standard_normal((8, V)) * 3).astype(np.float32)
    logits[3, 10:20] = logits[3].max() + 1  # ties at the maximum
    out["logits"] = logits
    out["argmax"] = np.array([ref.L.ref_argmax(np.ascontiguousarray(r), V) for r in logits], np.int32)
    params = [(1.0, 0, 1.0), (0.7, 0, 1.0), (1.3, 0, 1.0), (1.0, 40, 1.0), (1.0, 0, 0.9), (0.8, 25, 0.7), (0.0, 0, 1.0)]
    out["dist_params"] = np.array(params, np.float64)
    out["dist"] = np.stack([np.stack([ref.distribution(r, *p) for r in logits]) for p in params])
    # sample_from with Rng(seed)
    seeds = np.arange(64, dtype=np.uint64) * 7 + 3
    probs = np.stack([ref.distribution(logits[i % 8], 1.0) for i in range(64)])
    probs[5, ::2] = 0.0  # zeros are skipped
    out["sample_probs"] = probs
    out["sample_seeds"] = seeds
    out["sample_uniforms"] = np.array([ref.uniforms(int(s), 1)[0] for s in seeds])
    out["sample_out"] = np.array([ref.L.ref_sample_from(np.ascontiguousarray(probs[i]), V, int(seeds[i]))
                                  for i in range(64)], np.int32)
    # verify_speculative: B sequences, k drafts, with drafter distributions and one-hot
    B, k, V = 24, 4, 512
    tl = (rng.standard_normal((B, k + 1, V)) * 3).astype(np.float32)
    dl = (tl[:, :k] + rng.standard_normal((B, k, V)) * 0.5).astype(np.float32)
    P = np.stack([np.stack([ref.distribution(tl[b, j], 1.0) for j in range(k + 1)]) for b in range(B)])
    Q = np.stack([np.stack([ref.distribution(dl[b, j], 1.0) for j in range(k)]) for b in range(B)])
    drafts = np.zeros((B, k), np.int32)
    for b in range(B):
        u = ref.uniforms(1000 + b, k)
        for j in range(k):
            drafts[b, j] = ref.L.ref_sample_from(np.ascontiguousarray(Q[b, j]), V, 1000 * b + j)
        drafts[b, :] = np.where(u < 0.1, rng.integers(0, V, k), drafts[b])  # some unlikely drafts
    vseeds = np.arange(B, dtype=np.uint64) + 500
    acc, nxt = ref.verify(P, drafts, Q, vseeds)
    acc1, nxt1 = ref.verify(P, drafts, None, vseeds)
    out.update(verify_V=np.int32(V), verify_tlogits=tl, verify_dlogits=dl, verify_P=P, verify_Q=Q, verify_drafts=drafts,
               verify_seeds=vseeds, verify_uniforms=np.stack([ref.uniforms(int(s), k + 1) for s in vseeds]),
               verify_accepted=acc, verify_next=nxt, verify_accepted_onehot=acc1, verify_next_onehot=nxt1)
    return out


def make_philox(orc: Oracle) -> dict:
    kat_ctr = np.array([[0, 0, 0, 0], [0xFFFFFFFF] * 4, [0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344]], np.uint32)
    kat_key = np.array([[0, 0], [0xFFFFFFFF] * 2, [0xA4093822, 0x299F31D0]], np.uint32)
    # Published Random123 known answers for philox4x32_10 (kat_vectors); the oracle reproduces them.
    kat_out = np.array([[0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8],
                        [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD],
                        [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]], np.uint32)
    for i in range(3):
        assert np.array_equal(orc.philox(kat_ctr[i], kat_key[i]), kat_out[i]), "Philox KAT mismatch"
    uni = np.array([orc.philox_uniform(0x1234ABCD5678, i, 7, 9, 11) for i in range(256)])
    w = orc.gen_weights(0, 3, 1000, 4096, 0.02)
    return dict(kat_ctr=kat_ctr, kat_key=kat_key, kat_out=kat_out, uniform_seed=np.uint64(0x1234ABCD5678),
                uniforms=uni, gen_weights=w)


def make_fixture(ref: Reference) -> dict:
    d = tempfile.mkdtemp(prefix="clm_fixture_")
    ref.write_fixture(d, seed=FIXTURE_SEED)
    V, H, hc = 256, 64, 4
    fpp = hc * H + H + hc
    prompt_rng = ref.uniforms(0, 16)
    prompt = np.floor(prompt_rng * 256).astype(np.int32)
    out = {"prompt": prompt, "plan_bounds": np.array(PLAN_BOUNDS, np.int32)}

    def generate(q: int, drafts_fn, n_new: int, tag: str):
        p = RefPipeline(ref, d, PLAN_BOUNDS, max_context=256, max_window=8, vocab=V, floats_per_position=fpp)
        wid, base, state = 0, 0, 0
        committed: list[int] = []
        toks_log, acc_log, logits_log, stage_log = [], [], [], []
        nxt = 0
        for off in range(0, len(prompt), 8):
            chunk = prompt[off:off + 8]
            wid += 1
            logits, stages = p.run(wid, base, state, chunk, want_stages=True)
            p.commit(wid, state, len(chunk))
            toks_log.append(np.pad(chunk, (0, 8 - len(chunk)), constant_values=-1))
            acc_log.append(len(chunk))
            logits_log.append(np.pad(logits, ((0, 8 - len(chunk)), (0, 0))))
            stage_log.append(np.pad(stages, ((0, 0), (0, 8 - len(chunk)), (0, 0))))
            base += len(chunk)
            state += 1
            committed += list(chunk)
            nxt = int(np.argmax(logits[len(chunk) - 1]))
        generated: list[int] = []
        while len(generated) < n_new:
            window = [nxt] + (list(drafts_fn(committed, q - 1)) if q > 1 else [])
            wid += 1
            logits, stages = p.run(wid, base, state, np.array(window, np.int32), want_stages=True)
            accepted = 1
            for i in range(len(window) - 1):
                if int(np.argmax(logits[i])) != window[i + 1]:
                    break
                accepted += 1
            p.commit(wid, state, accepted)
            toks_log.append(np.pad(np.array(window, np.int32), (0, 8 - len(window)), constant_values=-1))
            acc_log.append(accepted)
            logits_log.append(np.pad(logits, ((0, 8 - len(window)), (0, 0))))
            stage_log.append(np.pad(stages, ((0, 0), (0, 8 - len(window)), (0, 0))))
            base += accepted
            state += 1
            committed += window[:accepted]
            generated += window[:accepted]
            nxt = int(np.argmax(logits[accepted - 1]))
        p.close()
        out[f"{tag}_tokens"] = np.stack(toks_log)
        out[f"{tag}_accepted"] = np.array(acc_log, np.int32)
        out[f"{tag}_logits"] = np.stack(logits_log).astype(np.float32)
        out[f"{tag}_stages"] = np.stack(stage_log).astype(np.float32)
        out[f"{tag}_generated"] = np.array(generated[:n_new], np.int32)
        return generated[:n_new]

    greedy = generate(1, None, 32, "greedy")
    continuation = np.array(list(prompt) + greedy, np.int32)
    out["scripted_reference"] = continuation
    generate(4, lambda committed, c: ref.scripted_draft(continuation, V, 1, 0.3, len(committed), c), 32, "spec")
    # MTP fixture drafter: one step for every previous token
    p = RefPipeline(ref, d, PLAN_BOUNDS, max_context=256, max_window=8, vocab=V, floats_per_position=fpp)
    out["mtp_step"] = np.array([p.mtp_step(t) for t in range(V)], np.int32)
    out["mtp_logits_0_7"] = np.stack([p.mtp_logits(t) for t in range(8)])
    p.close()
    return out


def main() -> None:
    ref, orc = Reference(), Oracle()
    np.savez_compressed(os.path.join(HERE, "codec.npz"), **make_codec(ref, orc))
    np.savez_compressed(os.path.join(HERE, "sampling.npz"), **make_sampling(ref))
    np.savez_compressed(os.path.join(HERE, "philox.npz"), **make_philox(orc))
    np.savez_compressed(os.path.join(HERE, "fixture.npz"), **make_fixture(ref))
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
