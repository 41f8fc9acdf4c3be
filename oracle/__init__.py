"""CPU oracle for the B200 self-play hot path — TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's (maxrlinder/card_playing_gym) algorithms on the
path: the plump field lookup, trunk conditioning, the KV-cached ragged decode of the
GQA trunk, the plump heads, masked sampling, undiscounted GAE, the PPO terms with
their gradient, and the dense value loss. Every function cites the reference
file:line it restates.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs
(``cpu_baseline`` and ``--impl reference``) may import this package, and only as the
checker or as the timed CPU baseline. The product path (``card_playing_gym_b200``)
never imports it and has no CPU fallback.

Parity pinning: the oracle is checked against (1) the reference's own golden
vectors ``tests/fixtures/plump_rl_v6_golden.npz`` with the rl-v6 release weights
(a CPU test that runs where the reference checkout is mounted), and (2) fixtures in
``tests/golden/`` that ``tests/golden/make_golden.py`` produced by running the
reference code itself on seeded inputs.
"""
