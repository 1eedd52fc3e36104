"""Serving benchmark harness (suite JSON schema v1, result JSON schema v2, summary/aggregate CSVs).

Behavioural parity with the reference's ``benchmarks/`` package: the same workload expansion,
arrival processes, closed-loop window rules, metric names and percentile definition, so results
are comparable line by line.  Additions: tensor-parallel / collective / load-format runtime keys
and B200 suites.
"""
