"""Oracles for the Local Attender -- test infrastructure only.

`local_attender_oracle` restates the reference with torch CPU ops;
`c_oracle` loads the double-precision C restatement (`make -C oracle`).
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs use
this package; the product never does.
"""
