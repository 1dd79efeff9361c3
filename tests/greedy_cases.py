"""Seeded greedy-selection cases shared by the oracle and GPU tests: the generator and case mix of
the reference's `greedy_select_matches_host_greedy_selection` (src/tests_conformance.rs:589-615),
restated -- xorshift64 with shifts 13/7/17 from 0x9e3779b9, coarse quarter-step scores so ties are
common, four special values planted per case, up to three short excluded ranges."""
import numpy as np

MASK = (1 << 64) - 1


class XorShift:
    def __init__(self, state=0x9E3779B9):
        self.state = state

    def __call__(self):
        s = self.state
        s ^= (s << 13) & MASK
        s ^= s >> 7
        s ^= (s << 17) & MASK
        self.state = s
        return s


def cases(rounds=40, widths=(151_936, 1000, 33, 7)):
    """Yields (logits [rows, cols] f32, row, excluded ranges, temperature) per round."""
    nxt = XorShift()
    specials = [np.float32("nan"), np.float32("inf"), np.float32("-inf"), np.float32(-0.0)]
    for rnd in range(rounds):
        cols = widths[rnd % 4]
        rows = 1 + rnd % 3
        data = np.array([((nxt() % 64) - 32.0) * 0.25 for _ in range(rows * cols)], np.float32)
        for _ in range(4):
            index = nxt() % (rows * cols)
            data[index] = specials[nxt() % 4]
        excluded = []
        for _ in range(nxt() % 4):
            start = nxt() % cols
            excluded.append((start, min(start + 1 + nxt() % 5, cols)))
        temperature = [0.0, 1.0, 0.7, 1.3][rnd % 4]
        row = nxt() % rows
        yield data.reshape(rows, cols), row, excluded, temperature


def host_greedy(scores, excluded, temperature):
    """The host rule in plain Python over f32 scalars (src/tests_conformance.rs:571-587)."""
    best = None
    for column, score in enumerate(np.asarray(scores, np.float32)):
        if not np.isfinite(score) or any(lo <= column < hi for lo, hi in excluded):
            continue
        s = score if temperature == 0.0 else np.float32(score / np.float32(temperature))
        if best is None or s > best[0]:
            best = (s, column)
    return None if best is None else best[1]
