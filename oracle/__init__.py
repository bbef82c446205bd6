"""CPU oracle package -- test and baseline infrastructure only.

``q4_oracle`` is the numpy restatement; ``cref`` loads the compiled C
restatement (``liboracle_q4.so``) and the reference's own compiled kernels
(``_ref/libsf_ref.so``).  The product package never imports this.
"""
