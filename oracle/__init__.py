"""CPU oracle (test infrastructure): numpy restatement of the reference's
pooling, coverage-mask and dense-masked attention algorithms. Used only by
tests/, __graft_entry__.smoke() and bench.py's CPU baseline."""
