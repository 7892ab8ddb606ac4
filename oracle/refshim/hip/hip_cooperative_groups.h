/* Empty stand-in: the reference's include/Cuda/PrefixSum.cuh includes the
 * cooperative-groups header but the host oracle uses none of it. */
#pragma once
