"""ORACLE package: CPU restatement of the DS-MeZO optimizer hot path.

Test infrastructure only (tests/, __graft_entry__.smoke(), bench.py's CPU baseline and
reference arm). The product package never imports it.
"""
from . import reference_ops  # noqa: F401
