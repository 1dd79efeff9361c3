"""Seeded Q8_0 packed weights and activations for the packed-weight tests, restating the
reference's generators (src/tests_conformance.rs:3325-3368): xorshift32 with shifts 13/17/5
seeded by seed * 2654435761 + 1, f16 scales between about 2^-9 and 2^-5, quants over -127..127;
activations ((i * 2246822519 + seed) mod 2001 - 1000) / 1000 with 32-bit wrapping."""
import numpy as np

M32 = 0xFFFFFFFF


def packed_q8(stored_rows, stored_cols, seed):
    """The 34-byte blocks of a stored_rows x stored_cols Q8_0 matrix, as uint8."""
    state = (seed * 2654435761 + 1) & M32

    def nxt():
        nonlocal state
        state ^= (state << 13) & M32
        state ^= state >> 17
        state ^= (state << 5) & M32
        return state

    blocks = stored_rows * stored_cols // 32
    out = np.empty((blocks, 34), np.uint8)
    for b in range(blocks):
        exponent = 6 + nxt() % 5
        d_bits = (exponent << 10) | (nxt() % 1024)
        out[b, 0] = d_bits & 0xFF
        out[b, 1] = d_bits >> 8
        out[b, 2:] = np.array([(nxt() % 255) - 127 for _ in range(32)], np.int64).astype(np.int8).view(np.uint8)
    return out.ravel()


def activations(rows, cols, seed):
    i = np.arange(rows * cols, dtype=np.uint64)
    v = ((i * np.uint64(2246822519) + np.uint64(seed)) & np.uint64(M32)) % np.uint64(2001)
    return ((v.astype(np.float32) - 1000.0) / 1000.0).reshape(rows, cols)


def checkpoint_blocks(rows, cols):
    """The closed-form table of the checkpoint-size test (src/tests_conformance.rs:4128-4150):
    d = 2^-7 (1 + (block mod 7) / 8), q = ((block * 31 + i * 7) mod 255) - 127; and its values."""
    blocks = rows * cols // 32
    b = np.arange(blocks, dtype=np.int64)
    d_bits = (8 << 10) | ((b % 7) << 7)
    out = np.empty((blocks, 34), np.uint8)
    out[:, 0] = (d_bits & 0xFF).astype(np.uint8)
    out[:, 1] = (d_bits >> 8).astype(np.uint8)
    i = np.arange(32, dtype=np.int64)
    q = ((b[:, None] * 31 + i[None, :] * 7) % 255) - 127
    out[:, 2:] = q.astype(np.int8).view(np.uint8)
    values = (q.astype(np.float32) * ((1.0 + (b % 7).astype(np.float32) / 8.0) / 128.0)[:, None]).reshape(rows, cols)
    return out.ravel(), values
