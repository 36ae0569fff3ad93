/* A plain C (C11) host of the provider's C ABI: it includes both public headers, links
 * libpcu_b200.so and calls the entry points that need no GPU (version, error strings, argument
 * checks that return before any device work, guarded-chain record validation).  Built and run by
 * tests/test_c_abi_host.py; exit status 0 means every check held. */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "pcu_b200.h"
#include "pcu_b200_graph.h"

static int failures = 0;

#define CHECK(cond)                                                      \
    do {                                                                 \
        if (!(cond)) {                                                   \
            fprintf(stderr, "check failed at line %d: %s\n", __LINE__, #cond); \
            ++failures;                                                  \
        }                                                                \
    } while (0)

int main(void) {
    CHECK(pcu_b200_abi_version() == PCU_B200_ABI_VERSION);
    CHECK(strcmp(pcu_b200_error_string(PCU_B200_OK), "ok") == 0);
    CHECK(strncmp(pcu_b200_error_string(PCU_B200_ERROR_WORKSPACE), "workspace", 9) == 0);

    /* arguments are checked before any device work */
    uint64_t status = 0;
    CHECK(pcu_b200_checked_binary(7, 0, PCU_B200_ADD, NULL, NULL, NULL, 0, 0, 0, &status, NULL) ==
          PCU_B200_ERROR_INVALID_ARGUMENT);
    CHECK(pcu_b200_strict_sgd(PCU_B200_F32, 0, NULL, NULL, NULL, 4, 0x3F000000u, NULL, NULL) ==
          PCU_B200_ERROR_INVALID_ARGUMENT);
    CHECK(pcu_b200_strict_matmul(PCU_B200_F32, 0, NULL, NULL, NULL, 0, 5, 5, 5, 5, 0, 0, NULL, 0, &status, NULL) ==
          PCU_B200_OK); /* an empty output is a successful no-op */
    CHECK(pcu_b200_guarded_checked_relu(PCU_B200_F32, 0, NULL, NULL, 4, NULL, 0, NULL) ==
          PCU_B200_ERROR_INVALID_ARGUMENT);
    /* the row-sharded all-gather's buffers: C, then a 256-byte flag block */
    CHECK(pcu_b200_peer_rows_bytes(PCU_B200_F32, 3, 5) == 512);
    CHECK(pcu_b200_mse_handoff_bytes() > 0 && pcu_b200_mse_handoff_bytes() % 256 == 0);
    /* a fused epilogue with more stages than the kernel carries is refused before any work */
    pcu_b200_epilogue_stage stages[PCU_B200_EPILOGUE_MAX + 1];
    memset(stages, 0, sizeof(stages));
    CHECK(pcu_b200_strict_matmul_epilogue(PCU_B200_F32, 0, NULL, NULL, NULL, 4, 4, 4, 4, 4, 0, 0, stages,
                                          PCU_B200_EPILOGUE_MAX + 1, NULL, 0, &status, NULL) ==
          PCU_B200_ERROR_INVALID_ARGUMENT);
    /* the split MSE needs its hand-off blocks and a call number */
    CHECK(pcu_b200_strict_mse_sgd_split(PCU_B200_F32, 0, NULL, NULL, 4, 0, 4, &status, NULL, 0, &status, NULL, NULL,
                                        NULL, 0, 0, 0, NULL, NULL, 0, 1, 1, NULL) == PCU_B200_ERROR_INVALID_ARGUMENT);
    pcu_b200_comm *comm = NULL;
    CHECK(pcu_b200_comm_init(NULL, 2, 0, &comm) == PCU_B200_ERROR_INVALID_ARGUMENT && comm == NULL);
    CHECK(pcu_b200_comm_free(NULL) == PCU_B200_OK);

    /* guarded-chain records: [fault word, disposition] per stage */
    const uint64_t ok = PCU_B200_STATUS_OK;
    const uint64_t fault = (900ull << 3) | PCU_B200_KIND_OVERFLOW;
    int outcome = -1;
    uint32_t stage = 99;
    uint64_t clean[4] = {ok, PCU_B200_CHAIN_EXECUTED, ok, PCU_B200_CHAIN_EXECUTED};
    CHECK(pcu_b200_chain_validate(clean, 2, NULL, &outcome, &stage) == PCU_B200_OK);
    CHECK(outcome == PCU_B200_CHAIN_SUCCEEDED && stage == 0);
    uint64_t faulted[6] = {ok, PCU_B200_CHAIN_EXECUTED, fault, PCU_B200_CHAIN_EXECUTED, ok, PCU_B200_CHAIN_SKIPPED};
    CHECK(pcu_b200_chain_validate(faulted, 3, NULL, &outcome, &stage) == PCU_B200_OK);
    CHECK(outcome == PCU_B200_CHAIN_FAULT && stage == 1);
    uint64_t extents[3] = {10, 900, 10};
    CHECK(pcu_b200_chain_validate(faulted, 3, extents, &outcome, &stage) == PCU_B200_OK);
    CHECK(outcome == PCU_B200_CHAIN_STAGE_DECODE && stage == 1);
    uint64_t late[4] = {fault, PCU_B200_CHAIN_EXECUTED, ok, PCU_B200_CHAIN_EXECUTED};
    CHECK(pcu_b200_chain_validate(late, 2, NULL, &outcome, &stage) == PCU_B200_OK);
    CHECK(outcome == PCU_B200_CHAIN_EXECUTED_AFTER_FAULT && stage == 1);

    if (failures) return 1;
    printf("c abi host ok\n");
    return 0;
}
