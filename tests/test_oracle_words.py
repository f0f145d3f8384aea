"""The C workload oracle against the reference's own definitions (CPU)."""
from __future__ import annotations

import numpy as np

import workload_oracle as W

MASK64 = (1 << 64) - 1


def reference_word(index, seed):
    """The reference test suite's host definition of the fill (tests/test_memory_read_contract.py:250-256)."""
    value = ((index ^ seed) + 0x9E3779B97F4A7C15) & MASK64
    value = ((value ^ (value >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    value = ((value ^ (value >> 27)) * 0x94D049BB133111EB) & MASK64
    return (value ^ (value >> 31)) & 0xFFFFFFFF


def reference_digest(workload, words, iterations, stride, offset, seed=7, blocks=2, threads=32):
    """Per-thread sums and their digest as the reference's GPU test states them (test_memory_read_contract.py:304-339)."""
    digest = 0
    region = words // blocks if workload == "l1" else words
    lanes = threads if workload == "l1" else blocks * threads
    for thread in range(blocks * threads):
        local = thread % threads if workload == "l1" else thread
        start = (thread // threads) * region if workload == "l1" else 0
        addresses = [start + ((local + it * lanes) * stride) % region for it in range(iterations)]
        thread_sum = sum(reference_word(a + offset // 4, seed) for a in addresses) & 0xFFFFFFFF
        digest = (digest * 1315423911 + thread_sum) & MASK64
    return digest


READ_CASES = (("l2", 1, 1, 1, 0), ("l2", 10, 7, 3, 4), ("l2", 2048, 2, 1, 32),
              ("l1", 2, 7, 1, 4), ("l1", 6, 5, 2, 4), ("l1", 4096, 1, 32, 0))


def test_fill_word_matches_reference_definition():
    rng = np.random.default_rng(3)
    for index in [0, 1, 2 ** 32 - 1, 2 ** 32, 2 ** 63 + 11] + [int(x) for x in rng.integers(0, 2 ** 62, 50)]:
        for seed in (0, 1, 7, 0x9E3779B9):
            assert W.lib().oracle_random_word(index ^ seed) == reference_word(index, seed)


def test_read_sum_digests_match_reference_cases():
    for workload, words, iterations, stride, offset in READ_CASES:
        slice_words = words // 2 if workload == "l1" else 0
        sums = W.read_sums(words if workload != "l1" else slice_words * 2, offset // 4, 7, 2, 32, stride, iterations,
                           slice_words=slice_words)
        assert W.sink_hash(sums) == reference_digest(workload, words, iterations, stride, offset)


def test_chase_links_form_one_cycle():
    for nodes, seed in ((1, 3), (7, 1), (1000, 42), (4099, 9)):
        links = W.chase_links(nodes, seed)
        seen, node = set(), 0
        for _ in range(nodes):
            seen.add(node)
            node = int(links[node])
        assert node == 0 and len(seen) == nodes


def test_sfu_initial_operands_are_half_open_unit_mantissas():
    for lane in range(0, 5000, 37):
        for chain in range(8):
            bits = W.lib().oracle_sfu_initial_bits(lane, 1, chain)
            x = np.frombuffer(np.uint32(bits).tobytes(), dtype=np.float32)[0]
            assert 0.5 <= x < 1.0


def test_lcg_fill_is_the_seeded_recurrence():
    for seed in (0, 11, 2 ** 40 + 5):
        words = W.lcg_words(1000, seed)
        x = seed & 0xFFFFFFFF
        for i in range(1000):
            assert int(words[i]) == x
            x = (1664525 * x + 1013904223) & 0xFFFFFFFF


def test_read_sums_over_an_explicit_payload_equal_the_random_word_sums():
    payload = np.array([W.lib().oracle_random_word(i ^ 11) for i in range(4096 + 8)], dtype=np.uint32)
    for unit in (1, 4):
        a = W.read_sums(4096, 8, 11, 4, 32, 3, 17, unit=unit)
        b = W.read_sums_of(payload, 4096, 8, 4, 32, 3, 17, unit=unit)
        assert np.array_equal(a, b)


def test_sfu_uniform_operands_lie_in_half_to_two():
    seen = []
    for lane in range(0, 20000, 7):
        for chain in range(4):
            bits = W.sfu_uniform_bits(lane, 3, chain)
            x = np.frombuffer(np.uint32(bits).tobytes(), dtype=np.float32)[0]
            m = W.lib().oracle_random_word(lane ^ 3 ^ ((chain + 1) * 0x9E3779B97F4A7C15 & MASK64)) >> 8
            assert x == np.float32(np.float32(m) * np.float32(1.5 / 16777216.0)) + np.float32(0.5)
            assert 0.5 <= x < 2.0
            seen.append(x)
    assert min(seen) < 0.52 and max(seen) > 1.98 and 0.3 < np.mean(np.array(seen) < 1.0) < 0.37
