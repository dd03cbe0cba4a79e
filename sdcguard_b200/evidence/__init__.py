"""Evidence: a scoped assessment of one recorded prefill/decode run of this engine (assessment.py) and a portable,
offline-verifiable bundle of what it was based on (bundle.py)."""
