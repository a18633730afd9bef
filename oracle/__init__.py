"""CPU restatement of the reference's hot-path arithmetic: the checker of tests/, smoke() and bench.py's CPU
baseline. Test infrastructure only; the product never imports it."""
