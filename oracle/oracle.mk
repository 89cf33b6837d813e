# Builds the C restatement of the reference (oracle/qnt_oracle.c) into oracle/_build/libqnt_oracle.so.
# TEST INFRASTRUCTURE ONLY.  Same float policy as the reference checker (oracle/Makefile): no FMA contraction.
HERE := $(dir $(abspath $(lastword $(MAKEFILE_LIST))))
OUT := $(HERE)_build
CC ?= gcc

all: $(OUT)/libqnt_oracle.so

$(OUT)/libqnt_oracle.so: $(HERE)qnt_oracle.c
	@mkdir -p $(OUT)
	$(CC) -O2 -std=gnu11 -fPIC -shared -ffp-contract=off -Wall -o $@ $< -lm

clean:
	rm -rf $(OUT)

.PHONY: all clean
