"""CPU oracle of ma_deform_attn -- test infrastructure only (see deform_oracle.py); the product never imports it."""
