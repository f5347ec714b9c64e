"""CPU oracle for the Gated DeltaNet path -- test infrastructure, not product.

``gdn_ref`` restates the reference's torch implementation
(solution/gdn_baseline_torch.py:12-91) in fp32 torch; ``c_oracle`` is the same
recurrence in C with OpenMP.  Only the tests, the smoke check and bench.py's
CPU legs import this package.
"""
