"""TEST INFRASTRUCTURE ONLY: CPU oracle for the authenticated KV transfer path.

Imported by tests/, ``__graft_entry__.smoke()`` and bench.py's CPU baseline /
reference arm as the checker.  ``secure_infer_b200`` never imports it.
"""
