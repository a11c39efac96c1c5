"""CPU oracle for the speculative-decoding path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of MicroServe's speculative step (reference
src/microserve/{sampling,speculative,model,cache}.py) with one change the
device needs: every random draw takes an explicit Philox uniform instead of
torch's CPU generator, so device and oracle can be compared draw for draw.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg (and
its ``--impl reference`` arm) may import this package, and only as the
checker or the timed CPU baseline -- never as a product code path.

Pinning: tests/golden/make_golden.py runs the unmodified reference (imported
from its source tree) to produce tests/golden/*.npz; tests/test_oracle.py
checks this restatement against those fixtures (logits, filtered
distributions, greedy streams and acceptance counts), and the Philox stream
against the Random123 known-answer vectors.
"""
