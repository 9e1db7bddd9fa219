"""CPU oracle package -- TEST INFRASTRUCTURE ONLY (tests/, smoke(), bench.py's CPU baseline)."""
