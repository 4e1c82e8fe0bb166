"""Host model of the one-shot all-reduce protocol of kernels/allreduce.cu.

Every (rank, CTA) pair is a thread; a rank's CTAs of one call finish before
its next call starts (stream order), ranks run freely against each other.
The shared arrays stand for the exchange areas: mailbox[rank][parity][src][i],
flags[rank][src][cta], epochs[rank][cta]. Each CTA owns the fixed element
range [c * CHUNK, (c + 1) * CHUNK) whatever n is, stores its chunk into every
peer's mailbox (parity = epoch & 1), raises its flag on every peer, waits for
the peers' flags and sums. Message sizes change from call to call, so a range
is used by some calls and skipped by others. The model is sequentially
consistent (it checks the protocol's reuse of mailbox slots, not the GPU
memory ordering, which the kernel gets from its system-scope fence and
release/acquire flags); random yields vary the interleaving. With CTA ranges
that follow n instead (a CTA count and chunk size computed from each
message), the model reads a later call's data within a few seeds: a range's
slot parity then mixes calls of different sizes.
"""
import random
import threading
import time

WORLD, CHUNK, CTAS = 4, 8, 4


def _run(calls, seed):
    rng = random.Random(seed)
    mailbox = [[[[None] * (CHUNK * CTAS) for _ in range(WORLD)] for _ in range(2)] for _ in range(WORLD)]
    flags = [[[0] * CTAS for _ in range(WORLD)] for _ in range(WORLD)]
    epochs = [[0] * CTAS for _ in range(WORLD)]
    parts = [[[rng.randint(-1000, 1000) for _ in range(n)] for n in calls] for _ in range(WORLD)]
    results = [[[None] * n for n in calls] for _ in range(WORLD)]
    barriers = [threading.Barrier(CTAS) for _ in range(WORLD)]
    errors = []

    def jitter(r):
        if r.random() < 0.3:
            time.sleep(0)

    def cta(rank, c):
        r = random.Random(seed * 1000 + rank * 10 + c)
        for k, n in enumerate(calls):
            lo, hi = c * CHUNK, min((c + 1) * CHUNK, n)
            if lo < n:
                e = epochs[rank][c] + 1
                par = e & 1
                for q in range(WORLD):
                    if q == rank:
                        continue
                    for i in range(lo, hi):
                        mailbox[q][par][rank][i] = (k, parts[rank][k][i])
                        jitter(r)
                for q in range(WORLD):
                    if q != rank:
                        flags[q][rank][c] = e
                        jitter(r)
                t0 = time.time()
                while any(flags[rank][q][c] < e for q in range(WORLD) if q != rank):
                    if time.time() - t0 > 20:
                        errors.append(f"rank {rank} cta {c} call {k}: wait timed out")
                        break
                    time.sleep(0)
                for i in range(lo, hi):
                    s = parts[rank][k][i]
                    for q in range(WORLD):
                        if q == rank:
                            continue
                        tag, v = mailbox[rank][par][q][i]
                        if tag != k:
                            errors.append(f"rank {rank} call {k} elem {i}: read call {tag}'s data from rank {q}")
                        s += v
                    results[rank][k][i] = s
                    jitter(r)
                epochs[rank][c] = e
            barriers[rank].wait()

    threads = [threading.Thread(target=cta, args=(rk, c)) for rk in range(WORLD) for c in range(CTAS)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors[:5]
    for k, n in enumerate(calls):
        want = [sum(parts[rk][k][i] for rk in range(WORLD)) for i in range(n)]
        for rk in range(WORLD):
            assert results[rk][k] == want, (rk, k)


def test_oneshot_protocol_fixed_ranges():
    # sizes that use 1..4 ranges, in an order that skips ranges between uses
    calls = [8, 32, 16, 8, 24, 32, 8, 8, 16, 32, 24, 8]
    for seed in range(3):
        _run(calls, seed)
