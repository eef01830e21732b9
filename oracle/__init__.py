"""CPU oracle for the GDN layer path (test infrastructure, never the product).

``gdn_oracle`` is the numpy restatement of the reference algorithms;
``cref`` loads the C restatement (``gdn_ref.c``) used for larger cases and for
the timed CPU baseline.
"""
